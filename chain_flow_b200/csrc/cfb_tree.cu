// cfb_tree.cu -- the tree-mode kernels around the drafting path (sm_100a): what the target model
// runs when it verifies a draft TREE instead of a chain.
//
//   tree_attn_merge_kernel   the tree-attention fix-up of a full-attention layer: every tree
//                            node attends to its own ancestors (the suffix), and that result is
//                            merged by log-sum-exp with the paged-prefix attention result.
//                            Restates the contract of the reference fork's suffix_merge
//                            (src/chain_flow/patches/vllm-0.25.1-chain-flow-tree.patch:5235-5540,
//                            its eager form _tree_suffix_eager :529-575 and vLLM's CUDA
//                            merge_attn_states op).
//
// Layout choices are this file's own; see each kernel.
#include <cuda_runtime.h>
#include <cuda_fp16.h>
#include <cuda_bf16.h>
#include <cstdint>
#include <cmath>

#include "../../include/cfb.h"
#include "cfb_common.cuh"

namespace {

__device__ __forceinline__ float tofl(__half x) { return __half2float(x); }
__device__ __forceinline__ float tofl(__nv_bfloat16 x) { return __bfloat162float(x); }
__device__ __forceinline__ void fromfl(__half& d, float x) { d = __float2half_rn(x); }
__device__ __forceinline__ void fromfl(__nv_bfloat16& d, float x) { d = __float2bfloat16_rn(x); }

// two elements <-> one 32-bit word
__device__ __forceinline__ float2 unpack2(uint32_t w, __half) {
  return __half22float2(*reinterpret_cast<const __half2*>(&w));
}
__device__ __forceinline__ float2 unpack2(uint32_t w, __nv_bfloat16) {
  return __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&w));
}
__device__ __forceinline__ uint32_t pack2(float a, float b, __half) {
  const __half2 h = __floats2half2_rn(a, b);
  return *reinterpret_cast<const uint32_t*>(&h);
}
__device__ __forceinline__ uint32_t pack2(float a, float b, __nv_bfloat16) {
  const __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
  return *reinterpret_cast<const uint32_t*>(&h);
}

// VPT consecutive elements of one row (VPT * 2 bytes: one vector access) as fp32
template <typename T, int VPT>
__device__ __forceinline__ void load_row(const T* p, float (&o)[VPT]) {
  static_assert(VPT == 2 || VPT == 4 || VPT == 8, "row slice");
  uint32_t w[VPT / 2];
  if constexpr (VPT == 8) {
    const uint4 r = *reinterpret_cast<const uint4*>(p);
    w[0] = r.x; w[1] = r.y; w[2] = r.z; w[3] = r.w;
  } else if constexpr (VPT == 4) {
    const uint2 r = *reinterpret_cast<const uint2*>(p);
    w[0] = r.x; w[1] = r.y;
  } else {
    w[0] = *reinterpret_cast<const uint32_t*>(p);
  }
#pragma unroll
  for (int i = 0; i < VPT / 2; ++i) {
    const float2 f = unpack2(w[i], T());
    o[2 * i] = f.x; o[2 * i + 1] = f.y;
  }
}
template <typename T, int VPT>
__device__ __forceinline__ void store_row(T* p, const float (&x)[VPT]) {
  uint32_t w[VPT / 2];
#pragma unroll
  for (int i = 0; i < VPT / 2; ++i) w[i] = pack2(x[2 * i], x[2 * i + 1], T());
  if constexpr (VPT == 8) *reinterpret_cast<uint4*>(p) = make_uint4(w[0], w[1], w[2], w[3]);
  else if constexpr (VPT == 4) *reinterpret_cast<uint2*>(p) = make_uint2(w[0], w[1]);
  else *reinterpret_cast<uint32_t*>(p) = w[0];
}

__device__ __forceinline__ float warp_max(float x) {
#pragma unroll
  for (int off = 16; off; off >>= 1) x = fmaxf(x, __shfl_xor_sync(0xffffffffu, x, off));
  return x;
}
__device__ __forceinline__ float warp_sum(float x) {
#pragma unroll
  for (int off = 16; off; off >>= 1) x += __shfl_xor_sync(0xffffffffu, x, off);
  return x;
}

// 32 partial sums per lane -> lane L ends with the warp-wide total of value L (a butterfly
// reduce-scatter: 31 shuffles for all 32 dot products instead of 5 per dot product).
__device__ __forceinline__ float reduce_scatter32(float (&v)[32]) {
  const int lane = threadIdx.x & 31;
#pragma unroll
  for (int s = 16; s >= 1; s >>= 1) {
    const bool upper = (lane & s) != 0;
#pragma unroll
    for (int i = 0; i < s; ++i) {
      const float send = upper ? v[i] : v[i + s];
      const float keep = upper ? v[i + s] : v[i];
      v[i] = keep + __shfl_xor_sync(0xffffffffu, send, s);
    }
  }
  return v[0];
}

// ---- tree attention suffix + log-sum-exp merge --------------------------------------------------
// One warp per (request s, query head h, tree node m); lane l owns head dims [l*VPT, l*VPT+VPT).
// The node's ancestor columns (mask byte 0, itself included) are compacted with ballots into a
// per-warp list. Their scores are computed 32 at a time: each lane forms the partial dot products
// of its dims with every ancestor key of the chunk, and one reduce-scatter leaves ancestor j's
// score on lane j. The softmax runs online across chunks (exact for any count; a depth-5 tree has
// at most 6 ancestors, one chunk). P.V accumulates in each lane's own dims, so it needs no
// reduction. The suffix result is rounded to the output dtype and back before the merge, as the
// eager path hands the merge a suffix already cast to the output dtype. Then
//   out = prefix * p_se / (p_se + s_se) + suffix * s_se / (p_se + s_se),  x_se = exp(x_lse - max)
// with a +inf lse read as -inf (vLLM's merge op), written at the node's query row.
constexpr int kAttnWarps = 4;
constexpr int kAttnMaxN = 128;             // nodes per request (4 mask words per lane)

struct AttnMergeArgs {
  const void* q; long long sq_t, sq_h;
  const void* k; long long sk_t, sk_h;
  const void* v; long long sv_t, sv_h;
  void* o; long long so_t, so_h;
  const void* po; long long spo_t, spo_h;
  const float* plse;                        // [H, S * N]
  const int64_t* idx;                       // [S, N] query row of each node
  const uint8_t* not_anc;                   // [S, N, N] 1 = masked out
  float scale;
  int S, N, H, rep;
};

template <typename T, int VPT>
__global__ void __launch_bounds__(kAttnWarps * 32, 1) tree_attn_merge_kernel(const AttnMergeArgs A) {
  __shared__ int s_col[kAttnWarps][kAttnMaxN];
  __shared__ long long s_row[kAttnMaxN];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int s = blockIdx.y;
  const int task = blockIdx.x * kAttnWarps + warp;          // over H * N
  const int h = task / A.N, m = task - (task / A.N) * A.N;
  const bool live = task < A.H * A.N;
  const long long mrow = (long long)s * A.N + m;            // this node's merge row
  // loads that depend on nothing: the node -> row table, the mask row, the prefix half
  for (int i = threadIdx.x; i < A.N; i += blockDim.x) s_row[i] = A.idx[(long long)s * A.N + i];
  uint32_t anc = 0u;                        // bit w: column w * 32 + lane is an ancestor
#pragma unroll
  for (int w = 0; w < kAttnMaxN / 32; ++w) {
    const int n = w * 32 + lane;
    if (live && n < A.N && A.not_anc[mrow * A.N + n] == 0) anc |= 1u << w;
  }
  float pr[VPT];
  float p_lse = 0.f;
  if (live) {
    load_row<T, VPT>(static_cast<const T*>(A.po) + mrow * A.spo_t + (long long)h * A.spo_h + lane * VPT, pr);
    p_lse = A.plse[(long long)h * ((long long)A.S * A.N) + mrow];
  }
  __syncthreads();
  if (!live) return;
  const long long rq = s_row[m];
  const int kh = h / A.rep;
  float qv[VPT];
  load_row<T, VPT>(static_cast<const T*>(A.q) + rq * A.sq_t + (long long)h * A.sq_h + lane * VPT, qv);
  // compact the ancestor columns, ascending
  int* col = s_col[warp];
  int c = 0;
  const unsigned below = (1u << lane) - 1u;
#pragma unroll
  for (int w = 0; w < kAttnMaxN / 32; ++w) {
    const bool ok = (anc >> w) & 1u;
    const unsigned b = __ballot_sync(0xffffffffu, ok);
    if (ok) col[c + __popc(b & below)] = w * 32 + lane;
    c += __popc(b);
  }
  __syncwarp();
  const T* kb = static_cast<const T*>(A.k) + (long long)kh * A.sk_h + lane * VPT;
  const T* vb = static_cast<const T*>(A.v) + (long long)kh * A.sv_h + lane * VPT;
  float mx = -INFINITY, den = 0.f;
  float acc[VPT];
#pragma unroll
  for (int d = 0; d < VPT; ++d) acc[d] = 0.f;
  for (int j0 = 0; j0 < c; j0 += 32) {
    const int cn = min(32, c - j0);
    float part[32];
#pragma unroll
    for (int j = 0; j < 32; ++j) {
      part[j] = 0.f;
      if (j < cn) {
        float kv[VPT];
        load_row<T, VPT>(kb + s_row[col[j0 + j]] * A.sk_t, kv);
#pragma unroll
        for (int d = 0; d < VPT; ++d) part[j] = fmaf(qv[d], kv[d], part[j]);
      }
    }
    const float dot = reduce_scatter32(part);               // every lane takes part
    const float sc = lane < cn ? dot * A.scale : -INFINITY;
    const float cmax = warp_max(sc);
    const float mnew = fmaxf(mx, cmax);
    const float e = lane < cn ? expf(sc - mnew) : 0.f;
    const float corr = (mx == -INFINITY) ? 0.f : expf(mx - mnew);
    den = den * corr + warp_sum(e);
#pragma unroll
    for (int d = 0; d < VPT; ++d) acc[d] *= corr;
    for (int j = 0; j < cn; ++j) {
      const float pj = __shfl_sync(0xffffffffu, e, j);
      float vv[VPT];
      load_row<T, VPT>(vb + s_row[col[j0 + j]] * A.sv_t, vv);
#pragma unroll
      for (int d = 0; d < VPT; ++d) acc[d] = fmaf(pj, vv[d], acc[d]);
    }
    mx = mnew;
  }
  // suffix output and lse (a node always attends to itself, so c >= 1 and den > 0)
  const float s_lse_raw = mx + logf(den);
  const float inv = 1.f / den;
  const float pl = (p_lse == INFINITY) ? -INFINITY : p_lse;
  const float sl = (s_lse_raw == INFINITY) ? -INFINITY : s_lse_raw;
  const float M = fmaxf(pl, sl);
  const float p_se = expf(pl - M), s_se = expf(sl - M);
  const float tot = p_se + s_se;
  const float p_scale = p_se / tot, s_scale = s_se / tot;
  float ov[VPT];
#pragma unroll
  for (int d = 0; d < VPT; ++d) {
    T r;
    fromfl(r, acc[d] * inv);
    ov[d] = fmaf(pr[d], p_scale, tofl(r) * s_scale);
  }
  store_row<T, VPT>(static_cast<T*>(A.o) + rq * A.so_t + (long long)h * A.so_h + lane * VPT, ov);
}

template <typename T>
cfb_status launch_attn_merge(const AttnMergeArgs& a, int D, cudaStream_t st) {
  const dim3 grid((a.H * a.N + kAttnWarps - 1) / kAttnWarps, a.S);
  switch (D) {
    case 64: tree_attn_merge_kernel<T, 2><<<grid, kAttnWarps * 32, 0, st>>>(a); break;
    case 128: tree_attn_merge_kernel<T, 4><<<grid, kAttnWarps * 32, 0, st>>>(a); break;
    case 256: tree_attn_merge_kernel<T, 8><<<grid, kAttnWarps * 32, 0, st>>>(a); break;
    default: return CFB_ERR_UNSUPPORTED;
  }
  return cfb_launch_status("tree_attn_merge_kernel");
}

}  // namespace

extern "C" cfb_status cfb_tree_attn_merge(const void* q, int64_t sq_t, int64_t sq_h, const void* k, int64_t sk_t,
                                          int64_t sk_h, const void* v, int64_t sv_t, int64_t sv_h, void* o,
                                          int64_t so_t, int64_t so_h, const void* prefix_out, int64_t spo_t,
                                          int64_t spo_h, const float* prefix_lse, const int64_t* idx,
                                          const uint8_t* not_anc, float scale, int S, int N, int H, int HKV,
                                          int D, int dtype, void* stream) {
  if (!q || !k || !v || !o || !prefix_out || !prefix_lse || !idx || !not_anc) return CFB_ERR_INVALID_ARG;
  if (S <= 0 || N <= 0 || H <= 0 || HKV <= 0) return CFB_ERR_INVALID_ARG;
  if (N > kAttnMaxN || H % HKV || (dtype != 1 && dtype != 2)) return CFB_ERR_UNSUPPORTED;
  // every row access is one vector of D / 32 elements per lane: rows start 16-byte aligned
  const int64_t strides[] = {sq_t, sq_h, sk_t, sk_h, sv_t, sv_h, so_t, so_h, spo_t, spo_h};
  for (int64_t s_ : strides)
    if (s_ <= 0 || (s_ * 2) % 16) return CFB_ERR_INVALID_ARG;
  const void* ptrs[] = {q, k, v, o, prefix_out};
  for (const void* p : ptrs)
    if (reinterpret_cast<uintptr_t>(p) % 16) return CFB_ERR_INVALID_ARG;
  AttnMergeArgs a{q, sq_t, sq_h, k, sk_t, sk_h, v, sv_t, sv_h, o, so_t, so_h, prefix_out, spo_t, spo_h,
                  prefix_lse, idx, not_anc, scale, S, N, H, H / HKV};
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  return dtype == 1 ? launch_attn_merge<__half>(a, D, st) : launch_attn_merge<__nv_bfloat16>(a, D, st);
}

// =================================================================================================
// Greedy tree verification: the target model's greedy continuation walked down the draft tree
// (the contract of the reference fork's tree_rejection_sample / tree_greedy_descent_kernel,
// src/chain_flow/patches/vllm-0.25.1-chain-flow-tree.patch:640-723). Request r owns n_r = cu_draft[r]
// - cu_draft[r - 1] draft nodes and the n_r + 1 logits rows [s0, s0 + n_r], s0 = cu_sampled[r] -
// (n_r + 1): row s0 scores the last committed token, row s0 + 1 + i tree node i. From the root the
// walk repeatedly takes the target's argmax token of the current row and moves to the FIRST child
// (in node order) of the current node whose draft token equals it; the accepted output is that path
// plus the argmax of the row where it stops (the bonus token).
//
// One launch does both halves. The argmax of every row (the HBM-bound part: the rows are whole
// vocabulary rows) is split over kVerifyChunks CTAs per row, each streaming its column range with
// 16-byte loads and publishing its (max, first index). A per-request arrival counter picks the CTA
// that finishes the request's last chunk; that CTA reduces the chunks of each of the request's rows
// in column order, stores the row argmaxes and walks the tree. Nobody waits, and the last arriver
// resets the counter, so the workspace is ready for the next launch (and for graph replay).
namespace {

constexpr int kVerifyThreads = 256;
constexpr int kVerifyChunks = 8;           // CTAs per logits row
constexpr int kVerifyMaxNodes = 1024;      // draft nodes per request (max_spec_len)

// torch.argmax order: larger value first, NaN above everything, ties to the lower index
__device__ __forceinline__ bool argmax_better(float v, int i, float bv, int bi) {
  const bool vn = v != v, bn = bv != bv;
  if (vn || bn) return vn && (!bn || i < bi);
  return v > bv || (v == bv && i < bi);
}

template <typename T>
__device__ __forceinline__ void argmax_span(const T* row, int c0, int c1, float& bv, int& bi) {
  // vector loads of 16 bytes where the span allows, scalar at its edges
  constexpr int E = 16 / (int)sizeof(T);
  const uintptr_t base = reinterpret_cast<uintptr_t>(row);
  int a = c0;
  while (a < c1 && ((base + (uintptr_t)a * sizeof(T)) & 15)) {
    if (((a - c0) % kVerifyThreads) == (int)threadIdx.x) {
      const float v = (float)row[a];
      if (argmax_better(v, a, bv, bi)) { bv = v; bi = a; }
    }
    ++a;
  }
  const int nvec = (c1 - a) / E;
  const uint4* vp = reinterpret_cast<const uint4*>(row + a);
  // kInFlight vectors per thread are loaded before any is compared, so the loads overlap
  constexpr int kInFlight = 4;
  for (int j0 = threadIdx.x; j0 < nvec; j0 += kInFlight * kVerifyThreads) {
    uint4 u[kInFlight];
#pragma unroll
    for (int q = 0; q < kInFlight; ++q) {
      const int j = j0 + q * kVerifyThreads;
      if (j < nvec) u[q] = __ldcs(vp + j);
    }
#pragma unroll
    for (int q = 0; q < kInFlight; ++q) {
      const int j = j0 + q * kVerifyThreads;
      if (j >= nvec) break;
      const T* t = reinterpret_cast<const T*>(&u[q]);
#pragma unroll
      for (int e = 0; e < E; ++e) {
        const float v = (float)t[e];
        const int c = a + j * E + e;
        if (argmax_better(v, c, bv, bi)) { bv = v; bi = c; }
      }
    }
  }
  for (int c = a + nvec * E + (int)threadIdx.x; c < c1; c += kVerifyThreads) {
    const float v = (float)row[c];
    if (argmax_better(v, c, bv, bi)) { bv = v; bi = c; }
  }
}

__device__ __forceinline__ float to_float(float x) { return x; }

struct VerifyGreedyArgs {
  const void* logits; long long ld; int V; int dtype;    // 0 fp32, 1 fp16, 2 bf16
  const int32_t* cu_draft; const int32_t* cu_sampled;     // [batch]
  const int32_t* draft_tokens; const int32_t* parents;    // [num_tokens]
  int batch, max_spec, num_rows;
  int32_t* out_tokens;    // [batch, max_spec + 1]
  int32_t* out_path;      // [batch, max_spec]
  int32_t* out_len;       // [batch]
  int32_t* row_argmax;    // [num_rows]
  float* part_v; int* part_i;    // [num_rows][kVerifyChunks]
  unsigned* counter;             // [batch]
  int* err;
};

// blockIdx.x = chunk, blockIdx.y = request, blockIdx.z = row of the request (grid.z = the largest
// n_r + 1; CTAs past a request's rows only count themselves in)
template <typename T>
__global__ void __launch_bounds__(kVerifyThreads) tree_verify_greedy_kernel(const VerifyGreedyArgs A) {
  __shared__ float s_v[kVerifyThreads / 32];
  __shared__ int s_i[kVerifyThreads / 32];
  __shared__ int s_last;
  const int r = blockIdx.y, ch = blockIdx.x, j = blockIdx.z;
  const int d0 = r ? A.cu_draft[r - 1] : 0, d1 = A.cu_draft[r];
  const int n = d1 - d0;
  const int s0 = A.cu_sampled[r] - (n + 1);
  // offsets that do not describe rows of this logits matrix are never dereferenced
  const bool sane = n >= 0 && n <= A.max_spec && s0 >= 0 && s0 + n < A.num_rows;
  const bool live = sane && j <= n;
  if (live) {
    const int row = s0 + j;
    const int c0 = (int)((long long)A.V * ch / kVerifyChunks), c1 = (int)((long long)A.V * (ch + 1) / kVerifyChunks);
    float bv = -INFINITY;
    int bi = 0x7fffffff;
    argmax_span(static_cast<const T*>(A.logits) + (long long)row * A.ld, c0, c1, bv, bi);
#pragma unroll
    for (int off = 16; off; off >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, bv, off);
      const int oi = __shfl_xor_sync(0xffffffffu, bi, off);
      if (argmax_better(ov, oi, bv, bi)) { bv = ov; bi = oi; }
    }
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (lane == 0) { s_v[warp] = bv; s_i[warp] = bi; }
    __syncthreads();
    if (threadIdx.x == 0) {
      for (int w = 1; w < kVerifyThreads / 32; ++w)
        if (argmax_better(s_v[w], s_i[w], bv, bi)) { bv = s_v[w]; bi = s_i[w]; }
      A.part_v[(long long)row * kVerifyChunks + ch] = bv;
      A.part_i[(long long)row * kVerifyChunks + ch] = bi;
    }
  }
  // count this CTA in; the request's last arriver finishes the rows and walks the tree
  if (threadIdx.x == 0) {
    __threadfence();
    const unsigned want = gridDim.z * (unsigned)kVerifyChunks;
    const unsigned prev = atomicAdd(A.counter + r, 1u);
    s_last = prev + 1 == want;
    if (s_last) { __threadfence(); A.counter[r] = 0u; }
  }
  __syncthreads();
  if (!s_last) return;
  // the request's last arriver: the whole CTA reduces the rows' chunks (a thread per row, chunks
  // in column order), stages the request's parents and draft tokens, then one warp walks the tree
  __threadfence();
  __shared__ int s_am[kVerifyMaxNodes + 1], s_par[kVerifyMaxNodes], s_tok[kVerifyMaxNodes];
  int32_t* ot = A.out_tokens + (long long)r * (A.max_spec + 1);
  int32_t* op = A.out_path + (long long)r * A.max_spec;
  for (int p = threadIdx.x; p <= A.max_spec; p += kVerifyThreads) ot[p] = -1;
  for (int p = threadIdx.x; p < A.max_spec; p += kVerifyThreads) op[p] = -1;
  if (!sane) {                            // inconsistent offsets: emit nothing, flag it
    if (threadIdx.x == 0) {
      A.out_len[r] = 0;
      if (A.err) atomicCAS(A.err, 0, cfb::DEV_BAD_INDEX);
    }
    return;
  }
  for (int jj = threadIdx.x; jj <= n; jj += kVerifyThreads) {
    const long long row = s0 + jj;
    float bv = __ldcg(A.part_v + row * kVerifyChunks);
    int bi = __ldcg(A.part_i + row * kVerifyChunks);
#pragma unroll
    for (int c = 1; c < kVerifyChunks; ++c) {
      const float v = __ldcg(A.part_v + row * kVerifyChunks + c);
      const int i = __ldcg(A.part_i + row * kVerifyChunks + c);
      if (argmax_better(v, i, bv, bi)) { bv = v; bi = i; }
    }
    A.row_argmax[row] = bi;
    s_am[jj] = bi;
  }
  for (int i = threadIdx.x; i < n; i += kVerifyThreads) { s_par[i] = A.parents[d0 + i]; s_tok[i] = A.draft_tokens[d0 + i]; }
  __syncthreads();
  if (threadIdx.x >= 32) return;
  const int lane = threadIdx.x;
  int cur = -1, pos = 0;
  for (;;) {
    const int tok = s_am[cur + 1];
    if (lane == 0) ot[pos] = tok;
    int nxt = -1;                         // the first child of cur carrying tok (node order)
    for (int i0 = 0; i0 < n && nxt < 0; i0 += 32) {
      const int i = i0 + lane;
      const unsigned hit = __ballot_sync(0xffffffffu, i < n && s_par[i] == cur && s_tok[i] == tok);
      if (hit) nxt = i0 + __ffs(hit) - 1;
    }
    if (nxt < 0 || pos >= A.max_spec) break;
    if (lane == 0) op[pos] = nxt;
    cur = nxt;
    ++pos;
  }
  if (lane == 0) A.out_len[r] = pos;
}

}  // namespace

extern "C" size_t cfb_tree_verify_workspace(int num_rows, int batch) {
  if (num_rows <= 0 || batch <= 0) return 0;
  const size_t parts = (size_t)num_rows * kVerifyChunks;
  return ((parts * 8 + 255) / 256) * 256 + (size_t)batch * 4;
}

extern "C" cfb_status cfb_tree_verify_greedy(const void* logits, int64_t ld, int num_rows, int V, int dtype,
                                             const int32_t* cu_num_draft, const int32_t* cu_num_sampled,
                                             const int32_t* draft_tokens, const int32_t* parents, int batch,
                                             int max_spec_len, int32_t* output_tokens, int32_t* accepted_path,
                                             int32_t* accepted_len, int32_t* row_argmax, void* ws,
                                             size_t ws_bytes, int* err, void* stream) {
  if (!logits || !cu_num_draft || !cu_num_sampled || !output_tokens || !accepted_path || !accepted_len ||
      !row_argmax || !ws)
    return CFB_ERR_INVALID_ARG;
  if (num_rows <= 0 || V <= 0 || batch <= 0 || max_spec_len < 0 || ld < V) return CFB_ERR_INVALID_ARG;
  if (max_spec_len > kVerifyMaxNodes) return CFB_ERR_UNSUPPORTED;
  if (max_spec_len > 0 && (!draft_tokens || !parents)) return CFB_ERR_INVALID_ARG;
  if (dtype < 0 || dtype > 2) return CFB_ERR_UNSUPPORTED;
  if ((reinterpret_cast<uintptr_t>(ws) & 255) || ws_bytes < cfb_tree_verify_workspace(num_rows, batch))
    return CFB_ERR_WORKSPACE;
  VerifyGreedyArgs a{};
  a.logits = logits; a.ld = ld; a.V = V; a.dtype = dtype;
  a.cu_draft = cu_num_draft; a.cu_sampled = cu_num_sampled; a.draft_tokens = draft_tokens; a.parents = parents;
  a.batch = batch; a.max_spec = max_spec_len; a.num_rows = num_rows;
  a.out_tokens = output_tokens; a.out_path = accepted_path; a.out_len = accepted_len; a.row_argmax = row_argmax;
  const size_t parts = (size_t)num_rows * kVerifyChunks;
  a.part_v = static_cast<float*>(ws);
  a.part_i = reinterpret_cast<int*>(static_cast<float*>(ws) + parts);
  a.counter = reinterpret_cast<unsigned*>(static_cast<char*>(ws) + ((parts * 8 + 255) / 256) * 256);
  a.err = err;
  const dim3 grid(kVerifyChunks, batch, max_spec_len + 1);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (dtype == 0) tree_verify_greedy_kernel<float><<<grid, kVerifyThreads, 0, st>>>(a);
  else if (dtype == 1) tree_verify_greedy_kernel<__half><<<grid, kVerifyThreads, 0, st>>>(a);
  else tree_verify_greedy_kernel<__nv_bfloat16><<<grid, kVerifyThreads, 0, st>>>(a);
  return cfb_launch_status("tree_verify_greedy_kernel");
}
