// cfb_wide.cu -- the batched ("wide") drafting path of libcfb.so: the tcgen05 GEMM and its host side.
//
// The persistent engine (cfb_engine.cu) drafts up to 8 requests per launch; its GEMM jobs hold at
// most 64 activation rows. Above that the flow's block GEMMs have hundreds of rows (B x 3 and
// B x 6 per Euler step and block), the weights are shared by every row, and the GEMMs become
// tensor-core work. The wide path runs them as TMA-fed tcgen05 GEMMs (cfb_wide_gemm.cuh) with
// fused epilogues, between small row-parallel kernels (LayerNorm, attention, beam).
#include <cuda_runtime.h>
#include <cudaTypedefs.h>
#include <mutex>
#include <vector>
#include "cfb_wide_gemm.cuh"

using namespace cfb;
using namespace cfb::wide;

namespace {

__device__ __forceinline__ void wide_err(int* err, int code) {
  if (err) atomicCAS(err, 0, code);
}

// ---- the epilogue of one 16-column slice of one accumulator row -------------------------------
template <int NV>
__device__ __forceinline__ void store_halves(__half* dst, const float (&v)[NV]) {
  uint4* d = reinterpret_cast<uint4*>(dst);
#pragma unroll
  for (int q = 0; q < NV / 8; ++q)
    d[q] = make_uint4(pack_half2(v[8 * q], v[8 * q + 1]), pack_half2(v[8 * q + 2], v[8 * q + 3]),
                      pack_half2(v[8 * q + 4], v[8 * q + 5]), pack_half2(v[8 * q + 6], v[8 * q + 7]));
}

// NV consecutive columns [col, col + NV) of one output row (NV a multiple of 4)
template <int NV>
__device__ __forceinline__ void epi_slice(const GemmProb& P, int sp, int row, int col, float (&v)[NV]) {
  if (P.bias && P.epi != EPI_PART && P.epi != EPI_PATH) {
    const float4* b4 = reinterpret_cast<const float4*>(P.bias + col);
#pragma unroll
    for (int q = 0; q < NV / 4; ++q) {
      const float4 b = b4[q];
      v[4 * q] += b.x; v[4 * q + 1] += b.y; v[4 * q + 2] += b.z; v[4 * q + 3] += b.w;
    }
  }
  switch (P.epi) {
    case EPI_F32:
    case EPI_PART: {
      float* o = static_cast<float*>(P.out) + (P.epi == EPI_PART ? (long long)sp * P.split_stride : 0) +
                 (long long)row * P.ldo + col;
      float4* o4 = reinterpret_cast<float4*>(o);
#pragma unroll
      for (int q = 0; q < NV / 4; ++q) o4[q] = make_float4(v[4 * q], v[4 * q + 1], v[4 * q + 2], v[4 * q + 3]);
      break;
    }
    case EPI_F16:
      store_halves(static_cast<__half*>(P.out) + (long long)row * P.ldo + col, v);
      break;
    case EPI_GELU16: {
#pragma unroll
      for (int i = 0; i < NV; ++i) v[i] = gelu_erf(v[i]);
      store_halves(static_cast<__half*>(P.out) + (long long)row * P.ldo + col, v);
      break;
    }
    case EPI_EULER: {
      const int b = row / P.chunk, c = row - b * P.chunk;
      float* z = static_cast<float*>(P.out) + ((long long)b * P.zrows + P.zstart + c) * P.ldo + col;
      float4* z4 = reinterpret_cast<float4*>(z);
#pragma unroll
      for (int q = 0; q < NV / 4; ++q) {
        float4 a = z4[q];
        a.x += P.dt * v[4 * q]; a.y += P.dt * v[4 * q + 1]; a.z += P.dt * v[4 * q + 2]; a.w += P.dt * v[4 * q + 3];
        z4[q] = a;
      }
      break;
    }
    case EPI_PATH: {
      const int64_t* lp = P.lastp + (long long)row * P.order;
      for (int j = 0; j < P.nlive; ++j) {
        if (lp[j] < 0) continue;
        const float4* b4 = reinterpret_cast<const float4*>(P.pbias + (long long)j * P.N + col);
#pragma unroll
        for (int q = 0; q < NV / 4; ++q) {
          const float4 b = b4[q];
          v[4 * q] += b.x; v[4 * q + 1] += b.y; v[4 * q + 2] += b.z; v[4 * q + 3] += b.w;
        }
      }
      float4* o4 = reinterpret_cast<float4*>(static_cast<float*>(P.out) + (long long)row * P.ldo + col);
#pragma unroll
      for (int q = 0; q < NV / 4; ++q) o4[q] = make_float4(v[4 * q], v[4 * q + 1], v[4 * q + 2], v[4 * q + 3]);
      break;
    }
    case EPI_HEADIN: {
      const int b = row / P.beams;
      const float4* p4 = reinterpret_cast<const float4*>(P.pred + ((long long)b * P.pred_rows + P.step) * P.N + col);
#pragma unroll
      for (int q = 0; q < NV / 4; ++q) {
        const float4 a = p4[q];
        v[4 * q] += a.x; v[4 * q + 1] += a.y; v[4 * q + 2] += a.z; v[4 * q + 3] += a.w;
      }
      store_halves(static_cast<__half*>(P.out) + (long long)row * P.ldo + col, v);
      break;
    }
    default:
      break;
  }
}

// ---- the GEMM kernel ----------------------------------------------------------------------------
// The fp32 logits of one accumulator row [col0, col0 + BN): online (max, sum exp) and the sorted
// top-`topb` (value, id) list, written to the row's list slot of this n tile. Per 16 columns: one
// max, 16 independent exponentials, and a list insertion only for a value that beats the list's
// current last entry (rare after the first columns).
__device__ __forceinline__ void head_row(const GemmProb& P, uint32_t tb, int nt, int row, bool live) {
  float m = -INFINITY, s = 0.f;
  float tv[kTopMaxW];
  int ti[kTopMaxW];
#pragma unroll
  for (int i = 0; i < kTopMaxW; ++i) { tv[i] = -INFINITY; ti[i] = 0x7fffffff; }
  float thr = -INFINITY;
  int thr_i = 0x7fffffff;
  for (int c0 = 0; c0 < BN; c0 += 16) {
    float v[16];
    tmem_ld16(tb + c0, v);                                    // every lane: .sync.aligned
    const int cb = nt * BN + c0;
    float cm = -INFINITY;
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      if (cb + i >= P.N) v[i] = -INFINITY;
      cm = fmaxf(cm, v[i]);
    }
    if (cm > m) { s *= __expf(m - cm); m = cm; }
    if (m > -INFINITY) {
      float cs = 0.f;
#pragma unroll
      for (int i = 0; i < 16; ++i) cs += __expf(v[i] - m);
      s += cs;
    }
    unsigned cand = 0;
#pragma unroll
    for (int i = 0; i < 16; ++i)
      if (better_w(v[i], cb + i + P.rowoff, thr, thr_i)) cand |= 1u << i;
    while (cand) {
      const int i = __ffs(cand) - 1;
      cand &= cand - 1;
      float xv = -INFINITY;
#pragma unroll
      for (int j = 0; j < 16; ++j) if (j == i) xv = v[j];
      int xi = cb + i + P.rowoff;
      if (!better_w(xv, xi, thr, thr_i)) continue;            // the list's last entry may have risen
#pragma unroll
      for (int q = 0; q < kTopMaxW; ++q) {
        if (q < P.topb && better_w(xv, xi, tv[q], ti[q])) {
          const float a = tv[q]; const int b = ti[q];
          tv[q] = xv; ti[q] = xi; xv = a; xi = b;
        }
      }
#pragma unroll
      for (int q = 0; q < kTopMaxW; ++q)
        if (q == P.topb - 1) { thr = tv[q]; thr_i = ti[q]; }
    }
  }
  if (live) {
    const int lw = 2 + 2 * P.topb;
    float* o = static_cast<float*>(P.out) + ((long long)row * P.n_tiles + nt) * lw;
    o[0] = m; o[1] = s;
#pragma unroll
    for (int q = 0; q < kTopMaxW; ++q)
      if (q < P.topb) { o[2 + q] = tv[q]; o[2 + P.topb + q] = __int_as_float(ti[q]); }
  }
}

// NH: 128-row M tiles per CTA (1, or 2 sharing each weight block; every problem of a launch
// must then have pair = 1), fixed at compile time so that the ring arithmetic is static.
template <int NH>
__global__ void __launch_bounds__(kGemmThreads, 1) wide_gemm_kernel(const __grid_constant__ GemmLaunch L) {
  constexpr uint32_t abytes = NH * kTileBytes;
  constexpr uint32_t stage = abytes + kWTileBytes;                       // 48 or 64 KiB
  constexpr int nst = (int)(kRingBytes / stage);                         // 4 or 3 stages
  constexpr uint32_t tcols = NH * BN;
  extern __shared__ uint8_t smraw[];
  uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smraw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(sm + kRingBytes);
  uint64_t* empty = full + kMaxStages;
  uint64_t* accf = empty + kMaxStages;
  uint32_t* tslot = reinterpret_cast<uint32_t*>(accf + 1);
  volatile int* sflag = reinterpret_cast<volatile int*>(tslot + 1);      // this CTA failed a wait
  volatile int* s_last = sflag + 1;                                      // split-K: this split is last

  int pi = 0;
  while (pi + 1 < L.nprob && (int)blockIdx.x >= L.p[pi + 1].cta0) ++pi;
  const GemmProb& P = L.p[pi];
  int t = (int)blockIdx.x - P.cta0;
  const int mp = t % P.m_pairs;
  t /= P.m_pairs;
  const int nt = t % P.n_tiles;
  const int sp = t / P.n_tiles;
  const int kb0 = sp * P.kb_per_split;
  const int nk = min(P.kblocks, kb0 + P.kb_per_split) - kb0;            // >= 1 (host guarantees)
  const int mt0 = NH * mp;                                              // first 128-row M tile
  const int nh = (NH == 2 && mt0 + 1 < P.m_tiles) ? 2 : 1;              // M tiles holding rows
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kMaxStages; ++s) { mbar_init(&full[s], 1); mbar_init(&empty[s], 1); }
    mbar_init(accf, 1);
    *sflag = 0;
    fence_mbar_init();
  }
  if (warp == 1) tmem_alloc(tslot, tcols);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tslot;

  if (warp == 0) {
    if (lane == 0) {
      prefetch_tmap(&P.ta);
      int issued = 0;
      for (int i = 0; i < nk; ++i) {
        const int s = i % nst;
        if (i >= nst && !mbar_wait(&empty[s], ((i / nst) - 1) & 1, nullptr, L.wait_ns)) { *sflag = 1; break; }
        if (*sflag) break;
        mbar_arrive_expect_tx(&full[s], stage);
        uint8_t* st = sm + s * stage;
        const int kb = kb0 + i;
        tma_load_2d(st, &P.ta, kb * BK, mt0 * BM, &full[s]);
        if (NH == 2) tma_load_2d(st + kTileBytes, &P.ta, kb * BK, (mt0 + 1) * BM, &full[s]);
        bulk_g2s(st + abytes, P.wt + ((long long)nt * P.kbt + kb) * (BN * BK), kWTileBytes, &full[s]);
        ++issued;
      }
      // copies still in flight land before the CTA may exit (bounded): after a failed wait the
      // MMA issuer may have stopped consuming them; the last nst copies are each stage's last use
      for (int i = max(0, issued - nst); i < issued; ++i) mbar_wait(&full[i % nst], (i / nst) & 1);
    }
  } else if (warp == 1) {
    if (lane == 0) {
      for (int i = 0; i < nk; ++i) {
        const int s = i % nst;
        if (!mbar_wait(&full[s], (i / nst) & 1, nullptr, L.wait_ns)) { *sflag = 1; break; }
        tc_fence_after();
        const uint32_t a = smem_u32(sm + s * stage), w = a + abytes;
#pragma unroll
        for (int k = 0; k < BK / 16; ++k) {
          const uint64_t wd = sw128_desc(w + k * 32);
          const uint32_t acc = (uint32_t)((i | k) != 0);
          tc_mma_f16(tmem, sw128_desc(a + k * 32), wd, kIdesc, acc);
          if (NH == 2) tc_mma_f16(tmem + BN, sw128_desc(a + kTileBytes + k * 32), wd, kIdesc, acc);
        }
        tc_commit(&empty[s]);
      }
      tc_commit(accf);       // arrives once every MMA issued above has completed
    }
  } else {
    const int lg = warp & 3;                                  // TMEM lanes 32*lg .. 32*lg+31
    // the issuer commits accf whether or not its loop completed, so this wait (default budget)
    // also keeps TMEM allocated until every MMA it issued has finished
    const bool ok = mbar_wait(accf, 0);
    tc_fence_after();
    if (!ok) *sflag = 1;
    const bool good = ok && *sflag == 0;
    if (P.epi == EPI_HEAD) {
      for (int h = 0; h < nh; ++h) {
        const int row = (mt0 + h) * BM + lg * 32 + lane;
        head_row(P, tmem + ((uint32_t)(lg * 32) << 16) + h * BN, nt, row, good && row < P.M);
      }
    } else if (P.splits > 1 && P.epi != EPI_PART) {
      // split-K of a non-partial epilogue: publish this split's tile; the split that arrives last
      // adds every split's tile in split order and applies the epilogue (nobody waits)
      const int tile = mp + P.m_pairs * nt;
      for (int h = 0; h < nh; ++h) {
        const int rl = h * BM + lg * 32 + lane;
        float* mine = P.fix_ws + (((long long)tile * P.splits + sp) * 2 * BM + rl) * BN;
        const uint32_t tb = tmem + ((uint32_t)(lg * 32) << 16) + h * BN;
        for (int c0 = 0; c0 < BN; c0 += 16) {
          float v[16];
          tmem_ld16(tb + c0, v);
          float4* o4 = reinterpret_cast<float4*>(mine + c0);
#pragma unroll
          for (int q = 0; q < 4; ++q) o4[q] = make_float4(v[4 * q], v[4 * q + 1], v[4 * q + 2], v[4 * q + 3]);
        }
      }
      consumer_sync(4 * 32);
      if (threadIdx.x == 2 * 32) {
        __threadfence();
        const int prev = atomicAdd(P.fix_cnt + tile, 1);
        const int last = prev == P.splits - 1;
        if (last) { P.fix_cnt[tile] = 0; __threadfence(); }
        *s_last = last;
      }
      consumer_sync(4 * 32);
      if (*s_last && good) {
        for (int h = 0; h < nh; ++h) {
          const int rl = h * BM + lg * 32 + lane;
          const int row = mt0 * BM + rl;
          if (row >= P.M) continue;
          const float* base = P.fix_ws + ((long long)tile * P.splits * 2 * BM + rl) * BN;
          for (int c0 = 0; c0 < BN; c0 += 16) {
            const int col = nt * BN + c0;
            if (col >= P.N) break;
            float v[16];
#pragma unroll
            for (int i = 0; i < 16; ++i) v[i] = 0.f;
            for (int q = 0; q < P.splits; ++q) {
              const float4* src = reinterpret_cast<const float4*>(base + (long long)q * 2 * BM * BN + c0);
#pragma unroll
              for (int z = 0; z < 4; ++z) {
                const float4 t4 = __ldcg(src + z);
                v[4 * z] += t4.x; v[4 * z + 1] += t4.y; v[4 * z + 2] += t4.z; v[4 * z + 3] += t4.w;
              }
            }
            epi_slice<16>(P, sp, row, col, v);
          }
        }
      }
    } else {
      for (int h = 0; h < nh; ++h) {
        const int row = (mt0 + h) * BM + lg * 32 + lane;
        const bool live = good && row < P.M;
        const uint32_t tb = tmem + ((uint32_t)(lg * 32) << 16) + h * BN;
        for (int c0 = 0; c0 < BN; c0 += 16) {
          float v[16];
          tmem_ld16(tb + c0, v);
          const int col = nt * BN + c0;
          if (live && col < P.N) epi_slice<16>(P, sp, row, col, v);
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, tcols);
  }
  if (threadIdx.x == 0 && *sflag) wide_err(L.err, DEV_TIMEOUT_FULL);
}

// ---- host: tensor maps and launches ----------------------------------------------------------
PFN_cuTensorMapEncodeTiled_v12000 g_encode = nullptr;
std::mutex g_wide_mu;
std::vector<int> g_gemm_attr_done;

cfb_status wide_init(int dev) {
  std::lock_guard<std::mutex> lk(g_wide_mu);
  if (!g_encode) {
    void* fn = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess || !fn)
      return cfb_launch_status("cudaGetDriverEntryPoint(cuTensorMapEncodeTiled)");
    g_encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
  }
  if ((int)g_gemm_attr_done.size() <= dev) g_gemm_attr_done.resize(dev + 1, 0);
  if (!g_gemm_attr_done[dev]) {
    if (cudaFuncSetAttribute(wide_gemm_kernel<1>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kGemmSmem) != cudaSuccess ||
        cudaFuncSetAttribute(wide_gemm_kernel<2>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kGemmSmem) != cudaSuccess)
      return cfb_launch_status("cudaFuncSetAttribute(wide_gemm_kernel)");
    g_gemm_attr_done[dev] = 1;
  }
  return CFB_OK;
}

// fp16 row-major [rows, k] with row stride ld (elements), tiles of 128 rows x 64 columns
cfb_status make_map(CUtensorMap* m, const void* base, long long rows, long long k, long long ld) {
  if (!base || rows <= 0 || k <= 0 || ld < k || (reinterpret_cast<uintptr_t>(base) & 15) || (ld * 2) % 16)
    return CFB_ERR_INVALID_ARG;
  cuuint64_t dims[2] = {(cuuint64_t)k, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)(ld * 2)};
  cuuint32_t box[2] = {(cuuint32_t)BK, (cuuint32_t)BM};
  cuuint32_t es[2] = {1, 1};
  CUresult r = g_encode(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void*>(base), dims, strides, box, es,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                        CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? CFB_OK : CFB_ERR_INVALID_ARG;
}

}  // namespace

namespace cfb {
namespace wide {

// Fill the shape part of one problem. K (the multiplied extent) must be a multiple of 64; every
// split gets at least one 64-column k block.
// W: tiled by cfb_wide_pack from a [N, ldw] matrix (ldw a multiple of 64); the GEMM multiplies its
// first K columns.
cfb_status gemm_prob(GemmProb& p, const void* A, long long lda, int M, const void* W, long long ldw, int N,
                     int K, int epi, int splits) {
  if (M <= 0 || N <= 0 || K <= 0 || K % BK || ldw % BK || K > ldw) return CFB_ERR_UNSUPPORTED;
  if (epi != EPI_HEAD && N % 16) return CFB_ERR_UNSUPPORTED;
  if (!W || (reinterpret_cast<uintptr_t>(W) & 15)) return CFB_ERR_INVALID_ARG;
  cfb_status st = make_map(&p.ta, A, M, K, lda);
  if (st != CFB_OK) return st;
  p.wt = static_cast<const __half*>(W);
  p.kbt = (int)(ldw / BK);
  p.M = M; p.N = N; p.kblocks = K / BK;
  p.m_tiles = (M + BM - 1) / BM;
  p.pair = 0;
  p.m_pairs = p.m_tiles;
  p.n_tiles = (N + BN - 1) / BN;
  splits = std::max(1, std::min(splits, p.kblocks));
  p.kb_per_split = (p.kblocks + splits - 1) / splits;
  p.splits = (p.kblocks + p.kb_per_split - 1) / p.kb_per_split;
  p.epi = epi;
  return CFB_OK;
}

cfb_status gemm_launch(GemmLaunch& L, cudaStream_t stream) {
  int total = 0;
  for (int i = 0; i < L.nprob; ++i) {
    L.p[i].cta0 = total;
    total += L.p[i].m_pairs * L.p[i].n_tiles * L.p[i].splits;
  }
  if (total <= 0) return CFB_OK;
  if (L.p[0].pair) wide_gemm_kernel<2><<<total, kGemmThreads, kGemmSmem, stream>>>(L);
  else wide_gemm_kernel<1><<<total, kGemmThreads, kGemmSmem, stream>>>(L);
  return cfb_launch_status("wide_gemm_kernel");
}

cfb_status init_device() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return cfb_launch_status("cudaGetDevice");
  return wide_init(dev);
}

}  // namespace wide
}  // namespace cfb

// =================================================================================================
// Row kernels of the wide path: LayerNorm (with the residual update in front of it), attention,
// the path-token gather and the beam step. All tensors are row-major.
namespace {

constexpr float kLnEps = 1e-5f;

enum LnMode : int {
  LN_PREP = 0,     // x32[b*S + i] = z[b, i] + pos[i] + (i >= start ? temb : 0), then LN
  LN_RESID = 1,    // x32 += bias + sum_s part[s], then LN
  LN_PLAIN32 = 2,  // LN of an fp32 matrix
  LN_PLAIN16 = 3,  // LN of an fp16 matrix
  LN_PATH = 4,     // x = sum_s part[s] + sum_{j < nlive, lastp[r][j] >= 0} pbias[j] (PathHead offsets)
  LN_POS = 5,      // x32[r] += pos[r % S] (learned positions after an in-projection), then LN
  LN_CAST = 6      // out = fp16(x32), no normalisation (an fp32 input of a GEMM)
};

struct LnSeg {
  int rows, row0, mode;
  float* x32;
  const __half* x16;
  const float* part; int nsplit; long long split_stride;
  const float* bias;
  const float* z; int zrows, S, start; const float* pos; const float* temb;
  __half* out;
  int cur_only, chunk;     // cur_only: write only rows i >= start, to out[b*chunk + i - start]
  const int64_t* lastp; int order, nlive; const float* pbias;    // LN_PATH
};
constexpr int kMaxLnSegs = 4;
struct LnLaunch { LnSeg s[kMaxLnSegs]; int nseg, D, rows; };

// One CTA (128 threads) per row; the row lives in registers (up to kLnMaxV float4 per thread)
// between the passes: residual update (bias + every split-K partial, loads all in flight),
// mean, centred variance, normalised fp16 output (nn.LayerNorm without its affine part, which
// is folded into the next Linear).
constexpr int kLnThreads = 128, kLnMaxV = 10, kLnMaxSplit = 8;
__device__ __forceinline__ float ln_block_sum(float v, float* red) {
  for (int off = 16; off > 0; off >>= 1) v += __shfl_xor_sync(0xffffffffu, v, off);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  __syncthreads();                                    // red[] free from a previous use
  if (lane == 0) red[warp] = v;
  __syncthreads();
  return (red[0] + red[1]) + (red[2] + red[3]);
}
__global__ void __launch_bounds__(kLnThreads) wide_ln_kernel(const __grid_constant__ LnLaunch L) {
  __shared__ float red[kLnThreads / 32];
  const int gr = blockIdx.x;
  int si = 0;
  while (si + 1 < L.nseg && gr >= L.s[si + 1].row0) ++si;
  const LnSeg& S = L.s[si];
  const int r = gr - S.row0;
  const int D = L.D;
  const int b = S.S > 0 ? r / S.S : 0, i = S.S > 0 ? r - b * S.S : 0;
  float4 x[kLnMaxV];
  float sum = 0.f;
#pragma unroll
  for (int v = 0; v < kLnMaxV; ++v) {
    const int c = (v * kLnThreads + threadIdx.x) * 4;
    float4 a = make_float4(0.f, 0.f, 0.f, 0.f);
    if (c < D) {
      if (S.mode == LN_PREP) {
        a = *reinterpret_cast<const float4*>(S.z + ((long long)b * S.zrows + i) * D + c);
        const float4 p = *reinterpret_cast<const float4*>(S.pos + (long long)i * D + c);
        a.x += p.x; a.y += p.y; a.z += p.z; a.w += p.w;
        if (i >= S.start) {
          const float4 t = *reinterpret_cast<const float4*>(S.temb + c);
          a.x += t.x; a.y += t.y; a.z += t.z; a.w += t.w;
        }
      } else if (S.mode == LN_RESID) {
        a = *reinterpret_cast<const float4*>(S.x32 + (long long)r * D + c);
        float4 acc = *reinterpret_cast<const float4*>(S.bias + c);
#pragma unroll
        for (int sp = 0; sp < kLnMaxSplit; ++sp)
          if (sp < S.nsplit) {
            const float4 q = *reinterpret_cast<const float4*>(S.part + sp * S.split_stride + (long long)r * D + c);
            acc.x += q.x; acc.y += q.y; acc.z += q.z; acc.w += q.w;
          }
        a.x += acc.x; a.y += acc.y; a.z += acc.z; a.w += acc.w;
      } else if (S.mode == LN_PLAIN32 || S.mode == LN_CAST) {
        a = *reinterpret_cast<const float4*>(S.x32 + (long long)r * D + c);
      } else if (S.mode == LN_POS) {
        a = *reinterpret_cast<const float4*>(S.x32 + (long long)r * D + c);
        const float4 p = *reinterpret_cast<const float4*>(S.pos + (long long)(r % S.S) * D + c);
        a.x += p.x; a.y += p.y; a.z += p.z; a.w += p.w;
        *reinterpret_cast<float4*>(S.x32 + (long long)r * D + c) = a;
      } else if (S.mode == LN_PATH) {
#pragma unroll
        for (int sp = 0; sp < kLnMaxSplit; ++sp)
          if (sp < S.nsplit) {
            const float4 q = *reinterpret_cast<const float4*>(S.part + sp * S.split_stride + (long long)r * D + c);
            a.x += q.x; a.y += q.y; a.z += q.z; a.w += q.w;
          }
        const int64_t* lp = S.lastp + (long long)r * S.order;
        for (int j = 0; j < S.nlive; ++j)
          if (lp[j] >= 0) {
            const float4 q = *reinterpret_cast<const float4*>(S.pbias + (long long)j * D + c);
            a.x += q.x; a.y += q.y; a.z += q.z; a.w += q.w;
          }
      } else {
        const uint2 h = *reinterpret_cast<const uint2*>(S.x16 + (long long)r * D + c);
        const float2 lo = unpack_half2(h.x), hi = unpack_half2(h.y);
        a = make_float4(lo.x, lo.y, hi.x, hi.y);
      }
      if (S.mode == LN_PREP || S.mode == LN_RESID) *reinterpret_cast<float4*>(S.x32 + (long long)r * D + c) = a;
    }
    x[v] = a;
    sum += (a.x + a.y) + (a.z + a.w);
  }
  if (S.mode == LN_CAST) {
#pragma unroll
    for (int v = 0; v < kLnMaxV; ++v) {
      const int c = (v * kLnThreads + threadIdx.x) * 4;
      if (c < D)
        *reinterpret_cast<uint2*>(S.out + (long long)r * D + c) =
            make_uint2(pack_half2(x[v].x, x[v].y), pack_half2(x[v].z, x[v].w));
    }
    return;
  }
  const float mean = ln_block_sum(sum, red) / (float)D;
  float var = 0.f;
#pragma unroll
  for (int v = 0; v < kLnMaxV; ++v) {
    const int c = (v * kLnThreads + threadIdx.x) * 4;
    if (c < D) {
      const float dx = x[v].x - mean, dy = x[v].y - mean, dz = x[v].z - mean, dw = x[v].w - mean;
      var += (dx * dx + dy * dy) + (dz * dz + dw * dw);
    }
  }
  const float rstd = rsqrtf(ln_block_sum(var, red) / (float)D + kLnEps);
  if (S.cur_only && i < S.start) return;
  const long long orow = S.cur_only ? (long long)b * S.chunk + (i - S.start) : r;
#pragma unroll
  for (int v = 0; v < kLnMaxV; ++v) {
    const int c = (v * kLnThreads + threadIdx.x) * 4;
    if (c < D)
      *reinterpret_cast<uint2*>(S.out + orow * D + c) =
          make_uint2(pack_half2((x[v].x - mean) * rstd, (x[v].y - mean) * rstd),
                     pack_half2((x[v].z - mean) * rstd, (x[v].w - mean) * rstd));
  }
}

// ---- attention: one CTA (4 warps) per (request, head, segment), one warp per query row -------------
// Lane l holds head-dimension chunks c = l + 32 t (8 halves each) of q, and of each key / value
// row as it streams past; the scores of the (at most kAttnMaxKeys) keys stay in registers.
constexpr int kAttnMaxKeys = 16, kAttnMaxChunks = 4;     // head dim <= 32 * 4 * 8 = 1024
struct AttnSeg {
  const __half* q; long long ldq; int qoff;
  const __half* k; const __half* v; long long ldkv; int koff, voff;
  int S, SK, causal;
  __half* out; long long ldo;
};
struct AttnLaunch { AttnSeg s[kMaxLnSegs]; int nseg, H, hd; float scale; };

__device__ __forceinline__ void h8_to_f(const uint4& u, float (&f)[8]) {
  const float2 a = unpack_half2(u.x), b = unpack_half2(u.y), c = unpack_half2(u.z), d = unpack_half2(u.w);
  f[0] = a.x; f[1] = a.y; f[2] = b.x; f[3] = b.y; f[4] = c.x; f[5] = c.y; f[6] = d.x; f[7] = d.y;
}

__global__ void __launch_bounds__(128) wide_attn_kernel(const __grid_constant__ AttnLaunch L) {
  const AttnSeg& A = L.s[blockIdx.y];
  const int b = blockIdx.x / L.H, h = blockIdx.x % L.H;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nch = L.hd / 8;
  for (int i = warp; i < A.S; i += 4) {
    float q[kAttnMaxChunks][8];
    const __half* qrow = A.q + ((long long)b * A.S + i) * A.ldq + A.qoff + h * L.hd;
#pragma unroll
    for (int t = 0; t < kAttnMaxChunks; ++t) {
      const int c = lane + 32 * t;
      if (c < nch) h8_to_f(*reinterpret_cast<const uint4*>(qrow + c * 8), q[t]);
      else {
#pragma unroll
        for (int z = 0; z < 8; ++z) q[t][z] = 0.f;
      }
    }
    const int nk = A.causal ? min(i + 1, A.SK) : A.SK;
    float sc[kAttnMaxKeys];
    float m = -INFINITY;
#pragma unroll
    for (int j = 0; j < kAttnMaxKeys; ++j) {
      sc[j] = -INFINITY;
      if (j < nk) {
        const __half* krow = A.k + ((long long)b * A.SK + j) * A.ldkv + A.koff + h * L.hd;
        float acc = 0.f;
#pragma unroll
        for (int t = 0; t < kAttnMaxChunks; ++t) {
          const int c = lane + 32 * t;
          if (c < nch) {
            float kf[8];
            h8_to_f(*reinterpret_cast<const uint4*>(krow + c * 8), kf);
#pragma unroll
            for (int z = 0; z < 8; ++z) acc += q[t][z] * kf[z];
          }
        }
        for (int off = 16; off > 0; off >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, off);
        sc[j] = acc * L.scale;
        m = fmaxf(m, sc[j]);
      }
    }
    float den = 0.f;
#pragma unroll
    for (int j = 0; j < kAttnMaxKeys; ++j) {
      sc[j] = j < nk ? expf(sc[j] - m) : 0.f;
      den += sc[j];
    }
    const float inv = 1.f / den;
    float o[kAttnMaxChunks][8];
#pragma unroll
    for (int t = 0; t < kAttnMaxChunks; ++t)
#pragma unroll
      for (int z = 0; z < 8; ++z) o[t][z] = 0.f;
#pragma unroll
    for (int j = 0; j < kAttnMaxKeys; ++j) {
      if (j < nk) {
        const __half* vrow = A.v + ((long long)b * A.SK + j) * A.ldkv + A.voff + h * L.hd;
        const float p = sc[j] * inv;
#pragma unroll
        for (int t = 0; t < kAttnMaxChunks; ++t) {
          const int c = lane + 32 * t;
          if (c < nch) {
            float vf[8];
            h8_to_f(*reinterpret_cast<const uint4*>(vrow + c * 8), vf);
#pragma unroll
            for (int z = 0; z < 8; ++z) o[t][z] += p * vf[z];
          }
        }
      }
    }
    __half* orow = A.out + ((long long)b * A.S + i) * A.ldo + h * L.hd;
#pragma unroll
    for (int t = 0; t < kAttnMaxChunks; ++t) {
      const int c = lane + 32 * t;
      if (c < nch)
        *reinterpret_cast<uint4*>(orow + c * 8) =
            make_uint4(pack_half2(o[t][0], o[t][1]), pack_half2(o[t][2], o[t][3]), pack_half2(o[t][4], o[t][5]),
                       pack_half2(o[t][6], o[t][7]));
    }
  }
}

// ---- initial latents and the head's starting state ------------------------------------------------
struct InitArgs {
  int mode;                   // cfb_init
  const __half* z0; const __half* ctx; float* z;
  int B, DL, C, D;
};
__global__ void wide_init_kernel(InitArgs a) {
  const long long n = (long long)a.B * a.DL * a.D;
  for (long long e = blockIdx.x * (long long)blockDim.x + threadIdx.x; e < n; e += (long long)gridDim.x * blockDim.x) {
    const int col = (int)(e % a.D);
    const long long bp = e / a.D;
    const int pos = (int)(bp % a.DL), b = (int)(bp / a.DL);
    float v;
    if (a.mode == CFB_INIT_GIVEN) {
      v = __half2float(a.z0[e]);
    } else {
      const float last = __half2float(a.ctx[((long long)b * a.C + a.C - 1) * a.D + col]);
      if (a.mode == CFB_INIT_REPEAT_LAST || a.C < 2) v = last;
      else v = last + (float)(pos + 1) * (last - __half2float(a.ctx[((long long)b * a.C + a.C - 2) * a.D + col]));
    }
    a.z[e] = v;
  }
}

struct HeadInitArgs {
  const int64_t* known0; int64_t* lastp; float* cum; int* prev; int B, Wmax, order;
};
// every row of request b starts from the committed token; only row 0 is a live beam
__global__ void wide_head_init_kernel(HeadInitArgs a) {
  const int r = blockIdx.x * blockDim.x + threadIdx.x;
  if (r >= a.B * a.Wmax) return;
  const int b = r / a.Wmax, w = r - b * a.Wmax;
  a.lastp[(long long)r * a.order] = a.known0[b];
  for (int j = 1; j < a.order; ++j) a.lastp[(long long)r * a.order + j] = -1;
  a.cum[r] = w == 0 ? 0.f : -INFINITY;
  a.prev[r] = -1;
}

// ---- path tokens -> path GEMM input, markov rows -> head input --------------------------------------
struct GatherArgs {
  const int64_t* lastp; int order, nlive, rows, D, rank;
  const __half* emb; __half* apath; long long lda;
  const __half* w1; __half* hin; long long ldh;
  int vocab; int* err;
};
// After a failed launch of the plan (err set) the path tokens may be stale or unset, so this
// kernel then does nothing; a token outside [0, vocab) is never dereferenced (it sets err).
__global__ void __launch_bounds__(128) wide_gather_kernel(GatherArgs a) {
  if (ld_volatile_int(a.err) != 0) return;
  const int r = blockIdx.x;
  const int64_t* lp = a.lastp + (long long)r * a.order;
  const int d8 = a.D / 8;
  for (int e = threadIdx.x; e < a.nlive * d8; e += blockDim.x) {
    const int j = e / d8, c = (e - j * d8) * 8;
    const int64_t tok = lp[j];
    uint4 val = make_uint4(0, 0, 0, 0);
    if (tok >= a.vocab) wide_err(a.err, DEV_BAD_INDEX);
    else if (tok >= 0) val = *reinterpret_cast<const uint4*>(a.emb + tok * a.D + c);
    *reinterpret_cast<uint4*>(a.apath + (long long)r * a.lda + (long long)j * a.D + c) = val;
  }
  const int64_t t0 = lp[0];
  if (t0 < 0 || t0 >= a.vocab) {
    if (threadIdx.x == 0) wide_err(a.err, DEV_BAD_INDEX);
    return;
  }
  for (int c = threadIdx.x * 8; c < a.rank; c += blockDim.x * 8)
    *reinterpret_cast<uint4*>(a.hin + (long long)r * a.ldh + a.D + c) =
        *reinterpret_cast<const uint4*>(a.w1 + t0 * a.rank + c);
}

// ---- beam step: one CTA (4 warps) per request ---------------------------------------------------------
constexpr int kBeamMaxRows = 16, kBeamMaxTop = 8;
struct BeamArgs {
  const float* lists; int ntiles, topb;        // lists [rows][ntiles][2 + 2 topb]
  int Wmax, fr, keep, order, depth, K, tree, N, base;
  float* cum; int64_t* lastp; int* prev;
  const int64_t* sl;
  int64_t* toks; int* bps;                     // chain: [K][B * Wmax]
  int64_t* tokens;                             // chain [B, K]; tree [B, 2N]
  int R; int* err;                             // shortlist rows; the plan's error word
};
// Like the gather, the beam step does nothing after a failed launch of the plan (its lists are
// then unset), and a list id outside the shortlist is never dereferenced (it sets err).
__global__ void __launch_bounds__(128) wide_beam_kernel(BeamArgs a) {
  if (ld_volatile_int(a.err) != 0) return;
  __shared__ float cv[kBeamMaxRows][kBeamMaxTop];
  __shared__ int ci[kBeamMaxRows][kBeamMaxTop];
  __shared__ int64_t oldlp[kBeamMaxRows][8];
  __shared__ float oldcum[kBeamMaxRows];
  __shared__ int oldprev[kBeamMaxRows];
  const int b = blockIdx.x, warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int lw = 2 + 2 * a.topb;
  for (int w = warp; w < a.fr; w += blockDim.x >> 5) {
    const int row = b * a.Wmax + w;
    const float* L0 = a.lists + (long long)row * a.ntiles * lw;
    // this lane's tiles: online (max, sumexp) and a sorted top list
    float m = -INFINITY, s = 0.f;
    float tv[kBeamMaxTop]; int ti[kBeamMaxTop];
#pragma unroll
    for (int q = 0; q < kBeamMaxTop; ++q) { tv[q] = -INFINITY; ti[q] = 0x7fffffff; }
    for (int t = lane; t < a.ntiles; t += 32) {
      const float* Lt = L0 + (long long)t * lw;
      const float mt = Lt[0], st = Lt[1];
      if (mt > m) { s = s * __expf(m - mt) + st; m = mt; }
      else if (mt > -INFINITY) s += st * __expf(mt - m);
      for (int j = 0; j < a.topb; ++j) {
        float xv = Lt[2 + j]; int xi = __float_as_int(Lt[2 + a.topb + j]);
#pragma unroll
        for (int q = 0; q < kBeamMaxTop; ++q)
          if (q < a.topb && better_w(xv, xi, tv[q], ti[q])) {
            const float u = tv[q]; const int k = ti[q]; tv[q] = xv; ti[q] = xi; xv = u; xi = k;
          }
      }
    }
    // warp: log-sum-exp (fixed xor tree), then topb rounds of an argmax over the lanes' heads
    for (int off = 16; off > 0; off >>= 1) {
      const float mo = __shfl_xor_sync(0xffffffffu, m, off), so = __shfl_xor_sync(0xffffffffu, s, off);
      const float M = fmaxf(m, mo);
      s = (M == -INFINITY) ? 0.f : s * __expf(m - M) + so * __expf(mo - M);
      m = M;
    }
    const float lse = m + logf(s);
    int head = 0;
    for (int q = 0; q < a.topb; ++q) {
      float v = -INFINITY; int id = 0x7fffffff;
#pragma unroll
      for (int z = 0; z < kBeamMaxTop; ++z) if (z == head) { v = tv[z]; id = ti[z]; }
      int own = lane;
      for (int off = 1; off < 32; off <<= 1) {
        const float vo = __shfl_xor_sync(0xffffffffu, v, off);
        const int io = __shfl_xor_sync(0xffffffffu, id, off), oo = __shfl_xor_sync(0xffffffffu, own, off);
        if (better_w(vo, io, v, id) || (vo == v && io == id && oo < own)) { v = vo; id = io; own = oo; }
      }
      if (lane == own) ++head;
      if (lane == 0) { cv[w][q] = v - lse; ci[w][q] = id; }
    }
  }
  for (int w = threadIdx.x; w < a.Wmax; w += blockDim.x) {
    const int row = b * a.Wmax + w;
    oldcum[w] = a.cum[row];
    oldprev[w] = a.prev[row];
    for (int j = 0; j < a.order; ++j) oldlp[w][j] = a.lastp[(long long)row * a.order + j];
  }
  __syncthreads();
  if (threadIdx.x != 0) return;
  // keep the best `keep` of the fr x topb extensions (value desc, then flat index asc)
  unsigned long long taken = 0ull;
  const int ncand = a.fr * a.topb;
  for (int k = 0; k < a.keep; ++k) {
    int best = -1; float bv = -INFINITY;
    for (int c = 0; c < ncand; ++c) {
      if (taken >> c & 1ull) continue;
      const float v = oldcum[c / a.topb] + cv[c / a.topb][c % a.topb];
      if (best < 0 || v > bv) { best = c; bv = v; }
    }
    taken |= 1ull << best;
    const int src = best / a.topb;
    const int sid = ci[src][best % a.topb];
    if (sid < 0 || sid >= a.R) { wide_err(a.err, DEV_BAD_INDEX); return; }
    const int64_t tok = a.sl[sid];
    const int row = b * a.Wmax + k;
    a.cum[row] = bv;
    int64_t* lp = a.lastp + (long long)row * a.order;
    lp[0] = tok;
    for (int j = 1; j < a.order; ++j) lp[j] = oldlp[src][j - 1];
    if (a.tree) {
      a.tokens[(long long)b * 2 * a.N + a.base + k] = tok;
      a.tokens[(long long)b * 2 * a.N + a.N + a.base + k] = oldprev[src];
      a.prev[row] = a.base + k;
    } else {
      a.toks[(long long)a.depth * gridDim.x * a.Wmax + row] = tok;
      a.bps[(long long)a.depth * gridDim.x * a.Wmax + row] = src;
    }
  }
  if (!a.tree && a.depth == a.K - 1) {      // walk the best beam back (first maximum wins)
    int idx = 0;
    for (int w = 1; w < a.keep; ++w) if (a.cum[b * a.Wmax + w] > a.cum[b * a.Wmax + idx]) idx = w;
    for (int st = a.K - 1; st >= 0; --st) {
      const long long o = (long long)st * gridDim.x * a.Wmax + b * a.Wmax + idx;
      a.tokens[(long long)b * a.K + st] = a.toks[o];
      idx = a.bps[o];
    }
  }
}

}  // namespace

// ---- weight packing for the wide GEMM ------------------------------------------------------------
namespace {
// one thread per 16-byte chunk of the packed matrix: block (nt, kb), row r, stored chunk c' holds
// source chunk c = c' ^ (r & 7) of row nt*128 + r, columns kb*64 + 8c .. +8 (zero past nout)
__global__ void wide_pack_kernel(const __half* __restrict__ w, long long ldw, int nout, int kbt, __half* __restrict__ dst,
                                 long long nchunks) {
  for (long long e = blockIdx.x * (long long)blockDim.x + threadIdx.x; e < nchunks; e += (long long)gridDim.x * blockDim.x) {
    const int cs = (int)(e & 7);
    const long long rowblk = e >> 3;                // (nt, kb, r)
    const int r = (int)(rowblk % BN);
    const long long blk = rowblk / BN;              // nt * kbt + kb
    const int kb = (int)(blk % kbt);
    const long long nt = blk / kbt;
    const long long n = nt * BN + r;
    const int c = cs ^ (r & 7);
    uint4 v = make_uint4(0, 0, 0, 0);
    if (n < nout) v = *reinterpret_cast<const uint4*>(w + n * ldw + (long long)kb * BK + c * 8);
    *reinterpret_cast<uint4*>(dst + e * 8) = v;
  }
}
}  // namespace

extern "C" size_t cfb_wide_packed_bytes(int nout, int k) {
  if (nout <= 0 || k <= 0 || k % BK) return 0;
  return (size_t)((nout + BN - 1) / BN) * BN * (size_t)k * sizeof(__half);
}

extern "C" cfb_status cfb_wide_pack(const void* w, int64_t ldw, int nout, int k, void* dst, void* stream) {
  if (!w || !dst || nout <= 0 || k <= 0 || ldw < k || (ldw % 8) || (reinterpret_cast<uintptr_t>(w) & 15) ||
      (reinterpret_cast<uintptr_t>(dst) & 15))
    return CFB_ERR_INVALID_ARG;
  if (k % BK) return CFB_ERR_UNSUPPORTED;
  const long long nchunks = (long long)((nout + BN - 1) / BN) * BN * (k / 8);
  const int blocks = (int)std::min<long long>((nchunks + 255) / 256, 1 << 16);
  wide_pack_kernel<<<blocks, 256, 0, static_cast<cudaStream_t>(stream)>>>(static_cast<const __half*>(w), ldw, nout,
                                                                        k / BK, static_cast<__half*>(dst), nchunks);
  return cfb_launch_status("wide_pack_kernel");
}

extern "C" cfb_status cfb_wide_gemm(const void* a, int64_t lda, const void* w, int64_t ldw, const float* bias,
                                    void* out, int64_t ldo, int M, int N, int K, int epi, int splits, int* err,
                                    void* stream) {
  if (!a || !w || !out || !err) return CFB_ERR_INVALID_ARG;
  if (epi != EPI_F32 && epi != EPI_F16 && epi != EPI_GELU16 && epi != EPI_PART) return CFB_ERR_UNSUPPORTED;
  if ((ldo % 4) || (reinterpret_cast<uintptr_t>(out) & 15) || (bias && (reinterpret_cast<uintptr_t>(bias) & 15)))
    return CFB_ERR_INVALID_ARG;
  cfb_status st = cfb::wide::init_device();
  if (st != CFB_OK) return st;
  GemmLaunch L{};
  L.nprob = 1;
  L.err = err;
  L.wait_ns = cfb::kWaitBudgetNs;
  GemmProb& p = L.p[0];
  if ((st = cfb::wide::gemm_prob(p, a, lda, M, w, ldw, N, K, epi, epi == EPI_PART ? splits : 1)) != CFB_OK) return st;
  p.bias = bias;
  p.out = out;
  p.ldo = ldo;
  p.split_stride = (long long)M * ldo;
  return cfb::wide::gemm_launch(L, static_cast<cudaStream_t>(stream));
}

// =================================================================================================
// The wide plan: the whole draft as a fixed list of launches over caller-owned buffers.
namespace {


struct Bump {
  char* base;
  size_t off = 0;
  template <class T>
  T* take(size_t n) {
    off = (off + 255) & ~size_t(255);
    T* p = base ? reinterpret_cast<T*>(base + off) : nullptr;
    off += n * sizeof(T);
    return p;
  }
};

enum StepKind { S_INIT, S_HEADINIT, S_LN, S_GEMM, S_ATTN, S_GATHER, S_BEAM };
struct Step { int kind, idx; };


}  // namespace

struct cfb_wide_plan {
  int dev = 0, nsm = 148;
  int* err = nullptr;
  std::vector<Step> steps;
  std::vector<GemmLaunch> gemms;
  std::vector<LnLaunch> lns;
  std::vector<AttnLaunch> attns;
  std::vector<GatherArgs> gathers;
  std::vector<BeamArgs> beams;
  InitArgs init{};
  HeadInitArgs hinit{};
  int batch = 0, head_rows = 0;
  int* fix_cnt = nullptr;      // split-K arrival counters: zero between launches
  size_t fix_cnt_bytes = 0;
  __half* hin = nullptr;       // head input: its padding columns stay zero
  size_t hin_bytes = 0;
  int kernel_launches = 0;
};

namespace {

// The launch shape of a grouped GEMM (the same for every problem of the group): split-K only
// when the group has fewer output tiles than SMs (one resident CTA per SM): as many splits as
// fill the SMs, each of at least 4 k blocks, at most 8, and at most 4 for a non-partial
// epilogue (whose last split reads every split's tile back from the fixup scratch fix_ws
// [fix_floats] with arrival counters fix_cnt [fix_tiles], shared by a plan's launches, which run
// one after another). A CTA covers one M tile; the kernel's two-tile mode (each weight block
// feeding two M tiles) measured slower on these shapes, where it halves an already short grid.
void shape_gemm(GemmLaunch& G, int nsm, float* fix_ws, size_t fix_floats, int* fix_cnt, int fix_tiles) {
  bool part = true, fix_ok = true;
  int tiles = 0, kmin = 1 << 30;
  for (int i = 0; i < G.nprob; ++i) {
    if (G.p[i].epi == EPI_HEAD) fix_ok = false;
    if (G.p[i].epi != EPI_PART) part = false;
    tiles += G.p[i].m_tiles * G.p[i].n_tiles;
    kmin = std::min(kmin, G.p[i].kblocks);
  }
  int bs = 1;
  if (tiles < nsm && (part || fix_ok)) {
    bs = std::min(std::max(1, nsm / tiles), std::max(1, kmin / 4));
    bs = std::min(bs, part ? 8 : 4);
  }
  size_t used = 0;
  int ctile = 0;
  for (int i = 0; i < G.nprob; ++i) {
    GemmProb& p = G.p[i];
    p.pair = 0;
    p.m_pairs = p.m_tiles;
    int s_ = std::min(bs, p.kblocks);
    const size_t per = (size_t)p.m_pairs * p.n_tiles * 2 * BM * BN;
    if (p.epi != EPI_PART) {
      while (s_ > 1 && used + per * s_ > fix_floats) --s_;
      if (s_ > 1 && ctile + p.m_pairs * p.n_tiles > fix_tiles) s_ = 1;
    }
    p.kb_per_split = (p.kblocks + s_ - 1) / s_;
    p.splits = (p.kblocks + p.kb_per_split - 1) / p.kb_per_split;
    if (p.epi != EPI_PART && p.splits > 1) {
      p.fix_ws = fix_ws + used;
      p.fix_cnt = fix_cnt + ctile;
      used += per * p.splits;
      ctile += p.m_pairs * p.n_tiles;
    }
  }
}

cfb_status wide_layout(const cfb_drafter* d, const cfb_run* r, Bump& bm, cfb_wide_plan* P) {
  using std::min;
  if (!d || !r) return CFB_ERR_INVALID_ARG;
  const int D = d->hidden, H = d->heads, Lb = d->layers, T = d->steps, DL = d->draft_len, CH = d->chunk;
  const int C = d->ctx_rows, E = d->n_experts, B = r->batch, order = d->path_order, rank = d->markov_rank;
  const bool flow = r->mode == CFB_MODE_FLOW || r->mode == CFB_MODE_CHAIN || r->mode == CFB_MODE_TREE;
  const bool tree = r->mode == CFB_MODE_TREE || r->mode == CFB_MODE_BEAM_TREE;
  const bool head = r->mode != CFB_MODE_FLOW;
  if (r->mode < CFB_MODE_FLOW || r->mode > CFB_MODE_BEAM_TREE) return CFB_ERR_INVALID_ARG;
  if (D <= 0 || D % 64 || H <= 0 || D % H || Lb <= 0 || T <= 0 || CH <= 0 || E <= 0 || E * CH != DL ||
      C <= 0 || B <= 0 || D > 4 * kLnThreads * kLnMaxV || (D / H) % 8 || D / H > 32 * 8 * kAttnMaxChunks ||
      C > kAttnMaxKeys || DL > kAttnMaxKeys)
    return CFB_ERR_UNSUPPORTED;
  if (r->ranks > 1) return CFB_ERR_UNSUPPORTED;           // the row-sharded head is engine-only
  if (r->twopass_m != 0) return CFB_ERR_UNSUPPORTED;      // so is the two-pass head
  if (flow && (r->init_mode < CFB_INIT_GIVEN || r->init_mode > CFB_INIT_DELTA || (r->init_mode == CFB_INIT_GIVEN && !r->z0)))
    return CFB_ERR_INVALID_ARG;
  if (!r->pred || (flow && !r->ctx) || (head && (!r->known0 || !r->tokens))) return CFB_ERR_INVALID_ARG;
  if (flow && (!d->experts || !d->experts[0].blocks)) return CFB_ERR_INVALID_ARG;
  const int hd = D / H, P2 = head ? d->path_up.nout : 0, FM = flow ? d->experts[0].blocks[0].ffn_up.nout / D : 0;
  const int Kh = head ? d->head.k : 0;     // head K: D + rank, padded with zero columns to a multiple of 64
  const int Wmax = tree ? std::max(1, r->tree_keep) : r->width;
  const int TB = tree ? r->tree_topb : r->width;
  const int K = tree ? min(r->depth, DL - 1) : r->depth;
  if (head) {
    if (Wmax < 1 || Wmax > kBeamMaxRows || TB < 1 || TB > kBeamMaxTop || TB > kTopMaxW || order < 1 || order > 8 ||
        K < 1 || K > DL - 1 || rank % 8 || d->head.nout != d->shortlist_rows || d->head.nout < TB ||
        d->head.k < D + rank || d->head.k % 64 ||
        d->path_offsets.nout != D || d->path_offsets.k != order * D || P2 % 64)
      return CFB_ERR_UNSUPPORTED;
    if ((long long)Wmax * TB > 64) return CFB_ERR_UNSUPPORTED;
  }
  // levels of the tree (nodes added per depth)
  std::vector<int> levels;
  int Ntree = 0;
  if (tree) {
    int fr = 1;
    for (int i = 0; i < K; ++i) { const int k = min(r->tree_keep, fr * TB); levels.push_back(k); Ntree += k; fr = k; }
  }

  int* err = bm.take<int>(64);
  // ---- flow buffers
  __half* ctxh = flow ? bm.take<__half>((size_t)B * C * D) : nullptr;
  std::vector<__half*> kvc(E * Lb, nullptr);
  std::vector<float*> x32(E), part(E);
  std::vector<__half*> xh(E), qkv(E), ao(E), qx(E), u(E), xc(E);
  const int nsm = P ? P->nsm : 148;
  const int SPL = 8;                                    // partial buffers: the largest split count
  // split-K fixup scratch, shared by the plan's launches (they run one after another): partial
  // tiles and per-tile arrival counters (zeroed once at creation; each launch leaves them zero)
  const size_t kFixFloats = (size_t)16 << 20;          // 64 MiB of partial tiles
  const int kFixTiles = 4096;
  float* fix_ws = bm.take<float>(kFixFloats);
  int* fix_cnt = bm.take<int>(kFixTiles);
  auto shape = [&](GemmLaunch& G) { shape_gemm(G, nsm, fix_ws, kFixFloats, fix_cnt, kFixTiles); };
  if (flow) {
    for (int i = 0; i < E * Lb; ++i) kvc[i] = bm.take<__half>((size_t)B * C * 2 * D);
    for (int e = 0; e < E; ++e) {
      const size_t rows = (size_t)B * (e + 1) * CH;
      x32[e] = bm.take<float>(rows * D);
      xh[e] = bm.take<__half>(rows * D);
      qkv[e] = bm.take<__half>(rows * 3 * D);
      ao[e] = bm.take<__half>(rows * D);
      qx[e] = bm.take<__half>(rows * D);
      u[e] = bm.take<__half>(rows * FM * D);
      part[e] = bm.take<float>((size_t)SPL * rows * D);
      xc[e] = bm.take<__half>((size_t)B * CH * D);
    }
  }
  // ---- head buffers
  const int BW = B * Wmax;
  const int ntiles = head ? (d->head.nout + BN - 1) / BN : 0;
  const int lw = 2 + 2 * TB;
  int64_t* lastp = nullptr; float* cum = nullptr; int* prev = nullptr; __half* apath = nullptr; float* hpart = nullptr;
  __half *hph = nullptr, *pm = nullptr, *hin = nullptr; float* lists = nullptr; int64_t* toks = nullptr; int* bps = nullptr;
  if (head) {
    lastp = bm.take<int64_t>((size_t)BW * order);
    cum = bm.take<float>(BW);
    prev = bm.take<int>(BW);
    apath = bm.take<__half>((size_t)BW * order * D);
    hpart = bm.take<float>((size_t)8 * BW * D);           // split-K partials of the path offsets
    hph = bm.take<__half>((size_t)BW * D);
    pm = bm.take<__half>((size_t)BW * P2);
    hin = bm.take<__half>((size_t)BW * Kh);
    lists = bm.take<float>((size_t)BW * ntiles * lw);
    toks = bm.take<int64_t>((size_t)K * BW);
    bps = bm.take<int>((size_t)K * BW);
  }
  if (!P) return CFB_OK;

  // ================================ the launch list ================================
  P->err = err;
  P->batch = B;
  cfb_status st;
  auto add_gemm = [&](GemmLaunch& L) {
    L.err = err;
    L.wait_ns = r->wait_budget_ns ? r->wait_budget_ns : kWaitBudgetNs;
    shape(L);
    P->gemms.push_back(L);
    P->steps.push_back({S_GEMM, (int)P->gemms.size() - 1});
  };
  P->fix_cnt = fix_cnt;
  P->fix_cnt_bytes = kFixTiles * sizeof(int);
  auto add_ln = [&](LnLaunch& L) {
    L.D = D;
    L.rows = 0;
    for (int i = 0; i < L.nseg; ++i) { L.s[i].row0 = L.rows; L.rows += L.s[i].rows; }
    P->lns.push_back(L);
    P->steps.push_back({S_LN, (int)P->lns.size() - 1});
  };
  const float dt = 1.f / (float)T;
  if (flow) {
    P->init = InitArgs{r->init_mode, static_cast<const __half*>(r->z0), static_cast<const __half*>(r->ctx), r->pred, B, DL, C, D};
    P->steps.push_back({S_INIT, 0});
    {
      LnLaunch L{};
      L.nseg = 1;
      LnSeg& s = L.s[0];
      s.rows = B * C; s.mode = LN_PLAIN16; s.x16 = static_cast<const __half*>(r->ctx); s.out = ctxh;
      add_ln(L);
    }
    // cross K/V of every (expert, block), once per draft
    GemmLaunch G{};
    for (int e = 0; e < E; ++e)
      for (int l = 0; l < Lb; ++l) {
        const cfb_linear& w = d->experts[e].blocks[l].cross_kv;
        GemmProb& p = G.p[G.nprob];
        if ((st = gemm_prob(p, ctxh, D, B * C, w.w, D, 2 * D, D, EPI_F16, 1)) != CFB_OK) return st;
        p.bias = w.bias; p.out = kvc[e * Lb + l]; p.ldo = 2 * D;
        if (++G.nprob == kMaxProbs) { add_gemm(G); G = GemmLaunch{}; }
      }
    if (G.nprob) add_gemm(G);
    for (int s = 0; s < T; ++s) {
      {
        LnLaunch L{};
        L.nseg = E;
        for (int e = 0; e < E; ++e) {
          LnSeg& g = L.s[e];
          g.rows = B * (e + 1) * CH; g.mode = LN_PREP; g.x32 = x32[e]; g.z = r->pred; g.zrows = DL; g.S = (e + 1) * CH;
          g.start = e * CH; g.pos = static_cast<const float*>(d->experts[e].pos_emb);
          g.temb = static_cast<const float*>(d->experts[e].temb) + (size_t)s * D; g.out = xh[e];
        }
        add_ln(L);
      }
      for (int l = 0; l < Lb; ++l) {
        auto gemm_e = [&](const cfb_linear cfb_block::*which, __half** A, int lda, int N, int K_, int epi, void** outs,
                          long long ldo, int split) -> cfb_status {
          GemmLaunch G2{};
          G2.nprob = E;
          for (int e = 0; e < E; ++e) {
            const cfb_linear& w = d->experts[e].blocks[l].*which;
            GemmProb& p = G2.p[e];
            cfb_status s2 = gemm_prob(p, A[e], lda, B * (e + 1) * CH, w.w, K_, N, K_, epi, split);
            if (s2 != CFB_OK) return s2;
            p.bias = w.bias; p.out = outs[e]; p.ldo = ldo;
            p.split_stride = (long long)B * (e + 1) * CH * D;
          }
          add_gemm(G2);
          return CFB_OK;
        };
        auto resid_ln = [&](const cfb_linear cfb_block::*which, bool last) {
          LnLaunch L{};
          L.nseg = E;
          const GemmLaunch& G3 = P->gemms.back();
          for (int e = 0; e < E; ++e) {
            LnSeg& g = L.s[e];
            g.rows = B * (e + 1) * CH; g.mode = LN_RESID; g.x32 = x32[e]; g.part = part[e];
            g.nsplit = G3.p[e].splits; g.split_stride = (long long)g.rows * D;
            g.bias = (d->experts[e].blocks[l].*which).bias;
            g.S = (e + 1) * CH; g.start = e * CH; g.chunk = CH;
            g.cur_only = last ? 1 : 0; g.out = last ? xc[e] : xh[e];
          }
          add_ln(L);
        };
        auto attn = [&](bool self_, int l_) {
          AttnLaunch A{};
          A.nseg = E; A.H = H; A.hd = hd; A.scale = 1.f / sqrtf((float)hd);
          for (int e = 0; e < E; ++e) {
            AttnSeg& g = A.s[e];
            g.S = (e + 1) * CH; g.out = ao[e]; g.ldo = D;
            if (self_) {
              g.q = qkv[e]; g.ldq = 3 * D; g.qoff = 0; g.k = g.v = qkv[e]; g.ldkv = 3 * D; g.koff = D; g.voff = 2 * D;
              g.SK = g.S; g.causal = 1;
            } else {
              g.q = qx[e]; g.ldq = D; g.qoff = 0; g.k = g.v = kvc[e * Lb + l_]; g.ldkv = 2 * D; g.koff = 0; g.voff = D;
              g.SK = C; g.causal = 0;
            }
          }
          P->attns.push_back(A);
          P->steps.push_back({S_ATTN, (int)P->attns.size() - 1});
        };
        void* o_qkv[kMaxProbs]; void* o_part[kMaxProbs]; void* o_qx[kMaxProbs]; void* o_u[kMaxProbs];
        for (int e = 0; e < E; ++e) { o_qkv[e] = qkv[e]; o_part[e] = part[e]; o_qx[e] = qx[e]; o_u[e] = u[e]; }
        if ((st = gemm_e(&cfb_block::qkv, xh.data(), D, 3 * D, D, EPI_F16, o_qkv, 3 * D, 1)) != CFB_OK) return st;
        attn(true, l);
        if ((st = gemm_e(&cfb_block::self_out, ao.data(), D, D, D, EPI_PART, o_part, D, 1)) != CFB_OK) return st;
        resid_ln(&cfb_block::self_out, false);
        if ((st = gemm_e(&cfb_block::cross_q, xh.data(), D, D, D, EPI_F16, o_qx, D, 1)) != CFB_OK) return st;
        attn(false, l);
        if ((st = gemm_e(&cfb_block::cross_out, ao.data(), D, D, D, EPI_PART, o_part, D, 1)) != CFB_OK) return st;
        resid_ln(&cfb_block::cross_out, false);
        if ((st = gemm_e(&cfb_block::ffn_up, xh.data(), D, FM * D, D, EPI_GELU16, o_u, FM * D, 1)) != CFB_OK) return st;
        {
          GemmLaunch G2{};
          G2.nprob = E;
          for (int e = 0; e < E; ++e) {
            const cfb_linear& w = d->experts[e].blocks[l].ffn_down;
            GemmProb& p = G2.p[e];
            if ((st = gemm_prob(p, u[e], FM * D, B * (e + 1) * CH, w.w, FM * D, D, FM * D, EPI_PART, 1)) != CFB_OK)
              return st;
            p.out = part[e]; p.ldo = D; p.split_stride = (long long)B * (e + 1) * CH * D;
          }
          add_gemm(G2);
        }
        resid_ln(&cfb_block::ffn_down, l == Lb - 1);
      }
      // out_proj of each expert's own rows + the Euler update of its chunk of z
      GemmLaunch G2{};
      G2.nprob = E;
      for (int e = 0; e < E; ++e) {
        const cfb_linear& w = d->experts[e].out_proj;
        GemmProb& p = G2.p[e];
        if ((st = gemm_prob(p, xc[e], D, B * CH, w.w, D, D, D, EPI_EULER, 1)) != CFB_OK) return st;
        p.bias = w.bias; p.out = r->pred; p.ldo = D; p.dt = dt; p.chunk = CH; p.zrows = DL; p.zstart = e * CH;
      }
      add_gemm(G2);
    }
  }
  if (head) {
    P->hinit = HeadInitArgs{r->known0, lastp, cum, prev, B, Wmax, order};
    P->steps.push_back({S_HEADINIT, 0});
    int base = 0;
    for (int dd = 0; dd < K; ++dd) {
      const int nlive = min(dd + 1, order);
      const int fr = tree ? (dd == 0 ? 1 : levels[dd - 1]) : Wmax;
      const int keep = tree ? levels[dd] : Wmax;
      P->gathers.push_back(GatherArgs{lastp, order, nlive, BW, D, rank, static_cast<const __half*>(d->embed), apath,
                                      (long long)order * D, static_cast<const __half*>(d->markov_w1), hin,
                                      (long long)Kh, d->vocab, err});
      P->steps.push_back({S_GATHER, (int)P->gathers.size() - 1});
      {
        GemmLaunch G{};
        G.nprob = 1;
        GemmProb& p = G.p[0];
        if ((st = gemm_prob(p, apath, (long long)order * D, BW, d->path_offsets.w, (long long)order * D, D, nlive * D,
                            EPI_PART, 1)) != CFB_OK)
          return st;
        p.out = hpart; p.ldo = D; p.split_stride = (long long)BW * D;
        add_gemm(G);
        LnLaunch L{};
        L.nseg = 1;
        LnSeg& g = L.s[0];
        g.rows = BW; g.mode = LN_PATH; g.part = hpart; g.nsplit = p.splits; g.split_stride = (long long)BW * D;
        g.lastp = lastp; g.order = order; g.nlive = nlive; g.pbias = d->path_offset_bias; g.out = hph;
        add_ln(L);
      }
      {
        GemmLaunch G{};
        G.nprob = 1;
        GemmProb& p = G.p[0];
        if ((st = gemm_prob(p, hph, D, BW, d->path_up.w, D, P2, D, EPI_GELU16, 1)) != CFB_OK) return st;
        p.bias = d->path_up.bias; p.out = pm; p.ldo = P2;
        add_gemm(G);
      }
      {
        GemmLaunch G{};
        G.nprob = 1;
        GemmProb& p = G.p[0];
        if ((st = gemm_prob(p, pm, P2, BW, d->path_down.w, P2, D, P2, EPI_HEADIN, 1)) != CFB_OK) return st;
        p.bias = d->path_down.bias; p.out = hin; p.ldo = Kh; p.pred = r->pred; p.beams = Wmax; p.pred_rows = DL;
        p.step = dd + 1;
        add_gemm(G);
      }
      {
        GemmLaunch G{};
        G.nprob = 1;
        GemmProb& p = G.p[0];
        if ((st = gemm_prob(p, hin, Kh, BW, d->head.w, Kh, d->head.nout, Kh, EPI_HEAD, 1)) != CFB_OK)
          return st;
        p.out = lists; p.topb = TB; p.rowoff = d->head_row0;
        add_gemm(G);
      }
      BeamArgs a{};
      a.lists = lists; a.ntiles = ntiles; a.topb = TB; a.Wmax = Wmax; a.fr = fr; a.keep = keep; a.order = order;
      a.depth = dd; a.K = K; a.tree = tree ? 1 : 0; a.N = Ntree; a.base = base; a.cum = cum; a.lastp = lastp; a.prev = prev;
      a.sl = d->shortlist; a.toks = toks; a.bps = bps; a.tokens = r->tokens;
      a.R = d->shortlist_rows; a.err = err;
      P->beams.push_back(a);
      P->steps.push_back({S_BEAM, (int)P->beams.size() - 1});
      base += keep;
    }
    P->head_rows = BW;
    P->hin = hin;
    P->hin_bytes = (size_t)BW * Kh * sizeof(__half);
  }
  P->kernel_launches = (int)P->steps.size();
  return CFB_OK;
}

cfb_status wide_run_steps(cfb_wide_plan* P, cudaStream_t st) {
  for (const Step& s : P->steps) {
    switch (s.kind) {
      case S_INIT: {
        const long long n = (long long)P->init.B * P->init.DL * P->init.D;
        const int blocks = (int)std::min<long long>((n + 255) / 256, 4L * P->nsm);
        wide_init_kernel<<<blocks, 256, 0, st>>>(P->init);
        break;
      }
      case S_HEADINIT:
        wide_head_init_kernel<<<(P->hinit.B * P->hinit.Wmax + 127) / 128, 128, 0, st>>>(P->hinit);
        break;
      case S_LN: {
        const LnLaunch& L = P->lns[s.idx];
        wide_ln_kernel<<<L.rows, kLnThreads, 0, st>>>(L);
        break;
      }
      case S_GEMM: {
        cfb_status r = gemm_launch(P->gemms[s.idx], st);
        if (r != CFB_OK) return r;
        continue;
      }
      case S_ATTN: {
        const AttnLaunch& A = P->attns[s.idx];
        wide_attn_kernel<<<dim3((unsigned)(P->batch * A.H), (unsigned)A.nseg), 128, 0, st>>>(A);
        break;
      }
      case S_GATHER: {
        const GatherArgs& g = P->gathers[s.idx];
        wide_gather_kernel<<<g.rows, 128, 0, st>>>(g);
        break;
      }
      case S_BEAM: {
        const BeamArgs& a = P->beams[s.idx];
        wide_beam_kernel<<<P->head_rows / a.Wmax, 128, 0, st>>>(a);
        break;
      }
    }
    cfb_status r = cfb_launch_status("wide path kernel");
    if (r != CFB_OK) return r;
  }
  return CFB_OK;
}

}  // namespace

// ---- the VAE bridge of the production drafter -----------------------------------------------------
// One side of the reference's TransformerHiddenVAE (encode: hidden -> mu; decode: latent ->
// hidden; transformer_hidden.py:51-67) as a launch list on the wide kernels: in-projection
// (+ bias, + learned positions), `layers` pre-LN encoder layers (bidirectional self-attention,
// GELU FFN), the final LayerNorm folded into the out-projection.
namespace {

cfb_status vae_layout(const cfb_vae_side* v, int B, int rows, int decode, const void* in, void* out, Bump& bm,
                      cfb_wide_plan* P) {
  if (!v || B <= 0 || rows <= 0) return CFB_ERR_INVALID_ARG;
  const int Hin = v->in_dim, Dw = v->width, Hout = v->out_dim, NL = v->layers, heads = v->heads;
  if (Hin % 64 || Dw % 64 || Hout % 16 || NL < 0 || heads <= 0 || Dw % heads || (Dw / heads) % 8 ||
      Dw / heads > 32 * 8 * kAttnMaxChunks || rows > kAttnMaxKeys || rows > v->max_len || Dw > 4 * kLnThreads * kLnMaxV ||
      (decode && Hin > 4 * kLnThreads * kLnMaxV))
    return CFB_ERR_UNSUPPORTED;
  if (!in || !out || !v->pos || !v->in_proj.w || !v->out_proj.w || (NL > 0 && !v->layer)) return CFB_ERR_INVALID_ARG;
  const int M = B * rows;
  const int FF = NL > 0 ? v->layer[0].ffn_up.nout : 0;
  int* err = bm.take<int>(64);
  const size_t kFixFloats = (size_t)8 << 20;           // 32 MiB of split-K fixup tiles
  const int kFixTiles = 1024;
  float* fix_ws = bm.take<float>(kFixFloats);
  int* fix_cnt = bm.take<int>(kFixTiles);
  __half* inh = decode ? bm.take<__half>((size_t)M * Hin) : nullptr;
  float* x32 = bm.take<float>((size_t)M * Dw);
  __half* xh = bm.take<__half>((size_t)M * Dw);
  __half* qkv = bm.take<__half>((size_t)M * 3 * Dw);
  __half* ao = bm.take<__half>((size_t)M * Dw);
  __half* u = bm.take<__half>((size_t)M * std::max(FF, 64));
  float* part = bm.take<float>((size_t)8 * M * Dw);
  if (!P) return CFB_OK;
  P->err = err;
  P->batch = B;
  cfb_status st;
  P->fix_cnt = fix_cnt;
  P->fix_cnt_bytes = kFixTiles * sizeof(int);
  auto add_gemm = [&](GemmLaunch& L, bool) {
    L.err = err;
    L.wait_ns = kWaitBudgetNs;
    shape_gemm(L, P->nsm, fix_ws, kFixFloats, fix_cnt, kFixTiles);
    P->gemms.push_back(L);
    P->steps.push_back({S_GEMM, (int)P->gemms.size() - 1});
  };
  auto add_ln = [&](LnLaunch& L, int D) {
    L.D = D;
    L.rows = 0;
    for (int i = 0; i < L.nseg; ++i) { L.s[i].row0 = L.rows; L.rows += L.s[i].rows; }
    P->lns.push_back(L);
    P->steps.push_back({S_LN, (int)P->lns.size() - 1});
  };
  const __half* A0 = static_cast<const __half*>(in);
  if (decode) {               // the latent arrives in fp32: an fp16 copy is the GEMM's input
    LnLaunch L{};
    L.nseg = 1;
    LnSeg& g = L.s[0];
    g.rows = M; g.mode = LN_CAST; g.x32 = const_cast<float*>(static_cast<const float*>(in)); g.out = inh;
    add_ln(L, Hin);
    A0 = inh;
  }
  {
    GemmLaunch G{};
    G.nprob = 1;
    GemmProb& p = G.p[0];
    if ((st = gemm_prob(p, A0, Hin, M, v->in_proj.w, v->in_proj.k, Dw, Hin, EPI_F32, 1)) != CFB_OK) return st;
    p.bias = v->in_proj.bias; p.out = x32; p.ldo = Dw;
    add_gemm(G, false);
    LnLaunch L{};
    L.nseg = 1;
    LnSeg& g = L.s[0];
    g.rows = M; g.mode = LN_POS; g.x32 = x32; g.pos = v->pos; g.S = rows; g.out = xh;
    add_ln(L, Dw);
  }
  auto resid = [&](const float* bias, int nsplit) {
    LnLaunch L{};
    L.nseg = 1;
    LnSeg& g = L.s[0];
    g.rows = M; g.mode = LN_RESID; g.x32 = x32; g.part = part; g.nsplit = nsplit; g.split_stride = (long long)M * Dw;
    g.bias = bias; g.out = xh;
    add_ln(L, Dw);
  };
  for (int l = 0; l < NL; ++l) {
    const cfb_vae_layer& ly = v->layer[l];
    {
      GemmLaunch G{};
      G.nprob = 1;
      GemmProb& p = G.p[0];
      if ((st = gemm_prob(p, xh, Dw, M, ly.qkv.w, ly.qkv.k, 3 * Dw, Dw, EPI_F16, 1)) != CFB_OK) return st;
      p.bias = ly.qkv.bias; p.out = qkv; p.ldo = 3 * Dw;
      add_gemm(G, false);
    }
    {
      AttnLaunch A{};
      A.nseg = 1; A.H = heads; A.hd = Dw / heads; A.scale = 1.f / sqrtf((float)(Dw / heads));
      AttnSeg& g = A.s[0];
      g.S = rows; g.SK = rows; g.causal = 0;
      g.q = qkv; g.ldq = 3 * Dw; g.qoff = 0; g.k = g.v = qkv; g.ldkv = 3 * Dw; g.koff = Dw; g.voff = 2 * Dw;
      g.out = ao; g.ldo = Dw;
      P->attns.push_back(A);
      P->steps.push_back({S_ATTN, (int)P->attns.size() - 1});
    }
    {
      GemmLaunch G{};
      G.nprob = 1;
      GemmProb& p = G.p[0];
      if ((st = gemm_prob(p, ao, Dw, M, ly.attn_out.w, ly.attn_out.k, Dw, Dw, EPI_PART, 1)) != CFB_OK) return st;
      p.out = part; p.ldo = Dw; p.split_stride = (long long)M * Dw;
      add_gemm(G, true);
      resid(ly.attn_out.bias, P->gemms.back().p[0].splits);
    }
    {
      GemmLaunch G{};
      G.nprob = 1;
      GemmProb& p = G.p[0];
      if ((st = gemm_prob(p, xh, Dw, M, ly.ffn_up.w, ly.ffn_up.k, FF, Dw, EPI_GELU16, 1)) != CFB_OK) return st;
      p.bias = ly.ffn_up.bias; p.out = u; p.ldo = FF;
      add_gemm(G, false);
    }
    {
      GemmLaunch G{};
      G.nprob = 1;
      GemmProb& p = G.p[0];
      if ((st = gemm_prob(p, u, FF, M, ly.ffn_down.w, ly.ffn_down.k, Dw, FF, EPI_PART, 1)) != CFB_OK) return st;
      p.out = part; p.ldo = Dw; p.split_stride = (long long)M * Dw;
      add_gemm(G, true);
      resid(ly.ffn_down.bias, P->gemms.back().p[0].splits);
    }
  }
  {
    GemmLaunch G{};
    G.nprob = 1;
    GemmProb& p = G.p[0];
    if ((st = gemm_prob(p, xh, Dw, M, v->out_proj.w, v->out_proj.k, Hout, Dw, decode ? EPI_F32 : EPI_F16, 1)) != CFB_OK)
      return st;
    p.bias = v->out_proj.bias; p.out = out; p.ldo = Hout;
    add_gemm(G, false);
  }
  P->kernel_launches = (int)P->steps.size();
  return CFB_OK;
}

}  // namespace

extern "C" cfb_status cfb_vae_workspace(const cfb_vae_side* v, int batch, int rows, int decode, size_t* bytes) {
  if (!bytes) return CFB_ERR_INVALID_ARG;
  Bump bm{nullptr};
  // shape checks need non-null I/O pointers: any non-null value serves the sizing pass
  cfb_status st = vae_layout(v, batch, rows, decode, reinterpret_cast<void*>(16), reinterpret_cast<void*>(16), bm,
                             nullptr);
  if (st != CFB_OK) return st;
  *bytes = bm.off + 256;
  return CFB_OK;
}

extern "C" cfb_status cfb_vae_create(const cfb_vae_side* v, int batch, int rows, int decode, const void* in, void* out,
                                     void* ws, size_t bytes, cfb_wide_plan** plan) {
  if (!ws || !plan || (reinterpret_cast<uintptr_t>(ws) & 255)) return CFB_ERR_INVALID_ARG;
  *plan = nullptr;
  size_t need = 0;
  cfb_status st = cfb_vae_workspace(v, batch, rows, decode, &need);
  if (st != CFB_OK) return st;
  if (bytes < need) return CFB_ERR_WORKSPACE;
  if ((st = cfb::wide::init_device()) != CFB_OK) return st;
  cfb_wide_plan* P = new cfb_wide_plan();
  cudaGetDevice(&P->dev);
  cudaDeviceGetAttribute(&P->nsm, cudaDevAttrMultiProcessorCount, P->dev);
  Bump bm{static_cast<char*>(ws)};
  st = vae_layout(v, batch, rows, decode, in, out, bm, P);
  if (st == CFB_OK && cudaMemset(P->err, 0, sizeof(int)) != cudaSuccess) st = cfb_launch_status("cudaMemset");
  if (st == CFB_OK && cudaMemset(P->fix_cnt, 0, P->fix_cnt_bytes) != cudaSuccess) st = cfb_launch_status("cudaMemset");
  if (st != CFB_OK) { delete P; return st; }
  *plan = P;
  return CFB_OK;
}

extern "C" cfb_status cfb_wide_workspace(const cfb_drafter* d, const cfb_run* r, size_t* bytes) {
  if (!bytes) return CFB_ERR_INVALID_ARG;
  Bump bm{nullptr};
  cfb_status st = wide_layout(d, r, bm, nullptr);
  if (st != CFB_OK) return st;
  *bytes = bm.off + 256;
  return CFB_OK;
}

extern "C" cfb_status cfb_wide_create(const cfb_drafter* d, const cfb_run* r, void* ws, size_t bytes,
                                      cfb_wide_plan** out) {
  if (!ws || !out || (reinterpret_cast<uintptr_t>(ws) & 255)) return CFB_ERR_INVALID_ARG;
  *out = nullptr;
  size_t need = 0;
  cfb_status st = cfb_wide_workspace(d, r, &need);
  if (st != CFB_OK) return st;
  if (bytes < need) return CFB_ERR_WORKSPACE;
  if ((st = cfb::wide::init_device()) != CFB_OK) return st;
  cfb_wide_plan* P = new cfb_wide_plan();
  cudaGetDevice(&P->dev);
  cudaDeviceGetAttribute(&P->nsm, cudaDevAttrMultiProcessorCount, P->dev);
  Bump bm{static_cast<char*>(ws)};
  st = wide_layout(d, r, bm, P);
  if (st == CFB_OK && cudaMemset(P->err, 0, sizeof(int)) != cudaSuccess) st = cfb_launch_status("cudaMemset");
  if (st == CFB_OK && P->hin && cudaMemset(P->hin, 0, P->hin_bytes) != cudaSuccess) st = cfb_launch_status("cudaMemset");
  if (st == CFB_OK && cudaMemset(P->fix_cnt, 0, P->fix_cnt_bytes) != cudaSuccess) st = cfb_launch_status("cudaMemset");
  if (st != CFB_OK) { delete P; return st; }
  *out = P;
  return CFB_OK;
}

extern "C" cfb_status cfb_wide_run(cfb_wide_plan* P, void* stream) {
  if (!P) return CFB_ERR_INVALID_ARG;
  return wide_run_steps(P, static_cast<cudaStream_t>(stream));
}

extern "C" cfb_status cfb_wide_error(cfb_wide_plan* P, int* device_error) {
  if (!P || !device_error) return CFB_ERR_INVALID_ARG;
  if (cudaMemcpy(device_error, P->err, sizeof(int), cudaMemcpyDeviceToHost) != cudaSuccess)
    return cfb_launch_status("cudaMemcpy(error word)");
  return CFB_OK;
}

extern "C" cfb_status cfb_wide_info(cfb_wide_plan* P, int* launches) {
  if (!P || !launches) return CFB_ERR_INVALID_ARG;
  *launches = P->kernel_launches;
  return CFB_OK;
}

extern "C" void cfb_wide_destroy(cfb_wide_plan* P) { delete P; }
