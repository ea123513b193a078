// cfb_gdn.cu -- tree-aware Gated-DeltaNet verification (sm_100a).
//
// Restates the recurrence of the reference's tree scan (src/chain_flow/kernels/tree_scan.py:29-78)
// and the fork's path-parallel verify kernels (patch tree_gdn.py:3285-3385,
// tree_gdn_verify.cu:4401-4562), node-serial instead of path-parallel: nodes arrive in BFS order
// (parent < child), so walking them in index order finds every parent state already written.
// Per node n with parent p (p < 0: the shared prefix state):
//     S = S_p * exp(g_n);  S += k_n (x) beta_n (v_n - S^T k_n);  o_n = S^T q_n
// q, k are L2-normalised as x / (||x|| + 1e-6) and q is scaled by Dk**-0.5 (tree_scan.py:25-27).
//
// One CTA per (request, head, 128 value columns). A thread owns one value column j and a quarter of the Dk = 128
// key rows (32 fp32 registers); the S^T k and S^T q column sums reduce over the 4 quarter
// threads with two shuffles. Every node state is written to `states` ([B,N,H,Dk,Dv] fp32,
// coalesced along j) and re-read from there as a parent: the same thread wrote it.
#include <cuda_runtime.h>
#include <cuda_fp16.h>
#include <cstdint>
#include <mutex>

#include "../../include/cfb.h"
#include "cfb_common.cuh"

namespace {

constexpr int kDk = 128;
constexpr int kQ = 4;                 // warps per CTA: each owns a quarter of the key rows
constexpr int kRowsPerThread = kDk / kQ;
constexpr int kColsPerBlock = 32;     // value columns per CTA (128 threads)
constexpr int kMaxNodes = 64;         // nodes per tree a CTA stages in shared memory
constexpr int kMinBlocks = 4;         // CTAs per SM the register budget is cut for
// dynamic shared memory of a launch over N-node trees: q, k (fp32) and 5 scalars per node
inline size_t gdn_smem(int N) { return (size_t)N * (2 * kDk + 5) * 4; }

// One CTA per (request, head, 32 value columns), 128 threads: warp w owns key rows
// [32w, 32w + 32) of the state and lane l the value column j = 32 * blockIdx.y + l, so every
// state load and store of a warp is one 128-byte row segment. Everything a node reads except
// its parent's state is staged in shared memory before the node loop: every node's q and k
// (fp32), their L2 norms, g, beta and the parent index. The S^T k and S^T q sums over the four
// row quarters go through shared memory (double-buffered by node parity: one barrier a node),
// and a thread keeps the state it just wrote in registers, so a node whose parent is the
// previous node reads no state from memory.
__global__ void __launch_bounds__(kColsPerBlock * kQ, kMinBlocks)
tree_gdn_kernel(const __half* __restrict__ q, const __half* __restrict__ k, const __half* __restrict__ v,
                const float* __restrict__ g, const float* __restrict__ beta, const int32_t* __restrict__ parent,
                const float* __restrict__ init, float* __restrict__ o, float* __restrict__ states, int N, int H,
                int Dv, int use_l2norm) {
  extern __shared__ float gsm[];
  float (*qs)[kDk] = reinterpret_cast<float (*)[kDk]>(gsm);
  float (*ks)[kDk] = reinterpret_cast<float (*)[kDk]>(gsm + (size_t)N * kDk);
  float* nq = gsm + (size_t)2 * N * kDk;
  float* nk = nq + N;
  float* gd = nk + N;
  float* bt = gd + N;
  int* pr = reinterpret_cast<int*>(bt + N);
  __shared__ float red[2][2][kQ][kColsPerBlock];    // [node parity][kv | o][row quarter][column]
  const int bh = blockIdx.x;
  const int b = bh / H, h = bh % H;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int j = blockIdx.y * kColsPerBlock + lane;     // value column
  const int k0 = warp * kRowsPerThread;                // first key row of this warp
  const float scale = rsqrtf((float)kDk);
  // stage q, k (fp16 -> fp32) of every node: 16-byte loads, all in flight together
  for (int e = tid; e < N * (kDk / 8); e += blockDim.x) {
    const int n = e / (kDk / 8), c = e - n * (kDk / 8);
    const size_t nh = ((size_t)b * N + n) * H + h;
    const uint4 qa = *reinterpret_cast<const uint4*>(q + nh * kDk + c * 8);
    const uint4 ka = *reinterpret_cast<const uint4*>(k + nh * kDk + c * 8);
    const __half2* q2 = reinterpret_cast<const __half2*>(&qa);
    const __half2* k2 = reinterpret_cast<const __half2*>(&ka);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float2 fq = __half22float2(q2[i]), fk = __half22float2(k2[i]);
      qs[n][c * 8 + 2 * i] = fq.x; qs[n][c * 8 + 2 * i + 1] = fq.y;
      ks[n][c * 8 + 2 * i] = fk.x; ks[n][c * 8 + 2 * i + 1] = fk.y;
    }
  }
  for (int n = tid; n < N; n += blockDim.x) {
    const size_t nh = ((size_t)b * N + n) * H + h;
    gd[n] = __expf(g[nh]);
    bt[n] = beta[nh];
    pr[n] = parent[(size_t)b * N + n];
  }
  __syncthreads();
  // L2 norms (x / (||x|| + 1e-6)), one warp per (node, q|k) row; q also takes Dk**-0.5
  for (int rr = warp; rr < 2 * N; rr += blockDim.x >> 5) {
    const int n = rr >> 1;
    const float* src = (rr & 1) ? ks[n] : qs[n];
    float ss = 0.f;
    for (int i = lane; i < kDk; i += 32) ss += src[i] * src[i];
    for (int off = 16; off > 0; off >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, off);
    if (lane == 0) {
      const float inv = use_l2norm ? 1.f / (sqrtf(ss) + 1e-6f) : 1.f;
      if (rr & 1) nk[n] = inv; else nq[n] = inv * scale;
    }
  }
  __syncthreads();
  const bool live = j < Dv;                            // Dv is a multiple of 32: whole warps
  float S[kRowsPerThread];
  int held = -2;                                       // the node whose state S holds
  for (int n = 0; n < N; ++n) {
    const size_t nh = ((size_t)b * N + n) * H + h;
    const int p = pr[n], par = n & 1;
    const float vj = live ? __half2float(v[nh * Dv + j]) : 0.f;
    if (p != held && live) {
      const float* src = (p < 0) ? init + ((size_t)b * H + h) * kDk * Dv
                                 : states + (((size_t)b * N + p) * H + h) * kDk * Dv;
#pragma unroll
      for (int i = 0; i < kRowsPerThread; ++i) S[i] = src[(size_t)(k0 + i) * Dv + j];
    }
    const float decay = gd[n], kn = nk[n], qn = nq[n];
    float kv = 0.f;
#pragma unroll
    for (int i = 0; i < kRowsPerThread; ++i) { S[i] *= decay; kv += S[i] * ks[n][k0 + i]; }
    red[par][0][warp][lane] = kv;
    __syncthreads();
    kv = (red[par][0][0][lane] + red[par][0][1][lane] + red[par][0][2][lane] + red[par][0][3][lane]) * kn;
    const float delta = (vj - kv) * bt[n];
    float on = 0.f;
    float* dst = states + nh * kDk * Dv;
#pragma unroll
    for (int i = 0; i < kRowsPerThread; ++i) {
      S[i] += (ks[n][k0 + i] * kn) * delta;
      on += S[i] * qs[n][k0 + i];
      if (live) __stcs(dst + (size_t)(k0 + i) * Dv + j, S[i]);
    }
    red[par][1][warp][lane] = on;
    __syncthreads();
    if (warp == 0 && live)
      o[nh * Dv + j] = (red[par][1][0][lane] + red[par][1][1][lane] + red[par][1][2][lane] + red[par][1][3][lane]) * qn;
    held = n;
  }
}

// trees of up to kMaxNodes nodes need more than the default 48 KB of dynamic shared memory
cfb_status gdn_smem_attr() {
  static std::mutex mu;
  static bool done[128] = {};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return cfb_launch_status("cudaGetDevice");
  std::lock_guard<std::mutex> lock(mu);
  if (dev >= 0 && dev < 128 && done[dev]) return CFB_OK;
  if (cudaFuncSetAttribute(tree_gdn_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)gdn_smem(kMaxNodes)) !=
      cudaSuccess)
    return cfb_launch_status("tree_gdn_kernel shared-memory attribute");
  if (dev >= 0 && dev < 128) done[dev] = true;
  return CFB_OK;
}

}  // namespace

extern "C" cfb_status cfb_tree_gdn(const void* q, const void* k, const void* v, const float* g,
                                   const float* beta, const int32_t* parent, const float* init,
                                   float* o, float* states, int B, int N, int H, int Dk, int Dv,
                                   int use_l2norm, void* stream) {
  if (!q || !k || !v || !g || !beta || !parent || !init || !o || !states) return CFB_ERR_INVALID_ARG;
  if (B <= 0 || N <= 0 || H <= 0) return CFB_ERR_INVALID_ARG;
  // >= 128 threads per CTA (every q/k element gets a loader thread, two warps for the norms)
  if (Dk != kDk || Dv <= 0 || Dv % kColsPerBlock || N > kMaxNodes) return CFB_ERR_UNSUPPORTED;
  const cfb_status sa = gdn_smem_attr();
  if (sa != CFB_OK) return sa;
  const dim3 grid(B * H, Dv / kColsPerBlock);
  tree_gdn_kernel<<<grid, kColsPerBlock * kQ, gdn_smem(N), static_cast<cudaStream_t>(stream)>>>(
      static_cast<const __half*>(q), static_cast<const __half*>(k), static_cast<const __half*>(v), g, beta,
      parent, init, o, states, N, H, Dv, use_l2norm);
  return cfb_launch_status("tree_gdn_kernel");
}

// ------------------------------------------------------------------------------------------
// No-allocation variant: the same kernel, with the per-node states (which it needs as scratch:
// every child re-reads its parent's state) held in a fixed device array of this library
// instead of a caller buffer. Nothing in the array has to start at zero: every node state is
// written before a child reads it, and the roots read `init`.
static __device__ __align__(256) float cfb_gdn_scratch[CFB_TREE_GDN_NOALLOC_MAX_FLOATS];

namespace {

constexpr int kMaxDevices = 128;
std::mutex g_scratch_mu;
float* g_scratch_ptr[kMaxDevices] = {};

// The device address of cfb_gdn_scratch on the current device, looked up once per device.
cfb_status scratch_for_current_device(float** out) {
  int dev = -1;
  if (cudaGetDevice(&dev) != cudaSuccess) {
    (void)cfb_launch_status("cudaGetDevice");
    return CFB_ERR_CUDA;
  }
  if (dev < 0 || dev >= kMaxDevices) return CFB_ERR_UNSUPPORTED;
  std::lock_guard<std::mutex> lock(g_scratch_mu);
  if (g_scratch_ptr[dev] == nullptr) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, cfb_gdn_scratch) != cudaSuccess) {
      (void)cfb_launch_status("cudaGetSymbolAddress(cfb_gdn_scratch)");
      return CFB_ERR_CUDA;
    }
    g_scratch_ptr[dev] = static_cast<float*>(p);
  }
  *out = g_scratch_ptr[dev];
  return CFB_OK;
}

}  // namespace

extern "C" cfb_status cfb_tree_gdn_noalloc(const void* q, const void* k, const void* v, const float* g,
                                           const float* beta, const int32_t* parent, const float* init,
                                           float* o, int B, int N, int H, int Dk, int Dv, int use_l2norm,
                                           void* stream) {
  if (!q || !k || !v || !g || !beta || !parent || !init || !o) return CFB_ERR_INVALID_ARG;
  if (B <= 0 || N <= 0 || H <= 0) return CFB_ERR_INVALID_ARG;
  if (Dk != kDk || Dv <= 0 || Dv % kColsPerBlock || N > kMaxNodes) return CFB_ERR_UNSUPPORTED;
  const unsigned long long need = (unsigned long long)B * N * H * Dk * Dv;
  if (need > (unsigned long long)CFB_TREE_GDN_NOALLOC_MAX_FLOATS) return CFB_ERR_WORKSPACE;
  float* scratch = nullptr;
  const cfb_status st = scratch_for_current_device(&scratch);
  if (st != CFB_OK) return st;
  const cfb_status sa = gdn_smem_attr();
  if (sa != CFB_OK) return sa;
  const dim3 grid(B * H, Dv / kColsPerBlock);
  tree_gdn_kernel<<<grid, kColsPerBlock * kQ, gdn_smem(N), static_cast<cudaStream_t>(stream)>>>(
      static_cast<const __half*>(q), static_cast<const __half*>(k), static_cast<const __half*>(v), g, beta,
      parent, init, o, scratch, N, H, Dv, use_l2norm);
  return cfb_launch_status("tree_gdn_kernel (no-alloc)");
}
