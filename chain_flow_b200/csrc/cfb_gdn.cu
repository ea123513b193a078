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
constexpr int kQ = 4;                 // threads per value column
constexpr int kRowsPerThread = kDk / kQ;

constexpr int kColsPerBlock = 128;     // value columns per CTA (512 threads)

__global__ void __launch_bounds__(kColsPerBlock * kQ)
tree_gdn_kernel(const __half* __restrict__ q, const __half* __restrict__ k, const __half* __restrict__ v, const float* __restrict__ g,
                                const float* __restrict__ beta, const int32_t* __restrict__ parent,
                                const float* __restrict__ init, float* __restrict__ o,
                                float* __restrict__ states, int N, int H, int Dv, int use_l2norm) {
  __shared__ float qs[kDk], ks[kDk];
  __shared__ float nrm[2];
  const int bh = blockIdx.x;
  const int b = bh / H, h = bh % H;
  const int tid = threadIdx.x;
  const int j = blockIdx.y * kColsPerBlock + (tid >> 2), qi = tid & 3;   // value column, key-row quarter
  const int k0 = qi * kRowsPerThread;
  const float scale = rsqrtf((float)kDk);
  float S[kRowsPerThread];
  for (int n = 0; n < N; ++n) {
    const size_t nh = ((size_t)b * N + n) * H + h;
    __syncthreads();
    if (tid < kDk) {
      qs[tid] = __half2float(q[nh * kDk + tid]);
      ks[tid] = __half2float(k[nh * kDk + tid]);
    }
    __syncthreads();
    if (tid < 64) {                              // warp 0: ||q||, warp 1: ||k||
      const float* src = (tid < 32) ? qs : ks;
      const int l = tid & 31;
      float s = 0.f;
      for (int i = l; i < kDk; i += 32) s += src[i] * src[i];
      for (int off = 16; off > 0; off >>= 1) s += __shfl_xor_sync(0xffffffffu, s, off);
      if (l == 0) nrm[tid >> 5] = use_l2norm ? 1.f / (sqrtf(s) + 1e-6f) : 1.f;
    }
    __syncthreads();
    if (j >= Dv) continue;
    const float qn = nrm[0] * scale, kn = nrm[1];
    const int p = parent[(size_t)b * N + n];
    const float* src = (p < 0) ? init + ((size_t)b * H + h) * kDk * Dv
                               : states + (((size_t)b * N + p) * H + h) * kDk * Dv;
    const float decay = __expf(g[nh]);
#pragma unroll
    for (int i = 0; i < kRowsPerThread; ++i) S[i] = src[(size_t)(k0 + i) * Dv + j] * decay;
    float kv = 0.f;
#pragma unroll
    for (int i = 0; i < kRowsPerThread; ++i) kv += S[i] * (ks[k0 + i] * kn);
    kv += __shfl_xor_sync(0xffffffffu, kv, 1);
    kv += __shfl_xor_sync(0xffffffffu, kv, 2);
    const float delta = (__half2float(v[nh * Dv + j]) - kv) * beta[nh];
    float on = 0.f;
    float* dst = states + nh * kDk * Dv;
#pragma unroll
    for (int i = 0; i < kRowsPerThread; ++i) {
      S[i] += (ks[k0 + i] * kn) * delta;
      on += S[i] * (qs[k0 + i] * qn);
      dst[(size_t)(k0 + i) * Dv + j] = S[i];
    }
    on += __shfl_xor_sync(0xffffffffu, on, 1);
    on += __shfl_xor_sync(0xffffffffu, on, 2);
    if (qi == 0) o[nh * Dv + j] = on;
  }
}

}  // namespace

extern "C" cfb_status cfb_tree_gdn(const void* q, const void* k, const void* v, const float* g,
                                   const float* beta, const int32_t* parent, const float* init,
                                   float* o, float* states, int B, int N, int H, int Dk, int Dv,
                                   int use_l2norm, void* stream) {
  if (!q || !k || !v || !g || !beta || !parent || !init || !o || !states) return CFB_ERR_INVALID_ARG;
  if (B <= 0 || N <= 0 || H <= 0) return CFB_ERR_INVALID_ARG;
  // >= 128 threads per CTA (every q/k element gets a loader thread, two warps for the norms)
  if (Dk != kDk || Dv <= 0 || Dv % 32 || (Dv > kColsPerBlock && Dv % kColsPerBlock)) return CFB_ERR_UNSUPPORTED;
  const int cols = Dv < kColsPerBlock ? Dv : kColsPerBlock;
  const dim3 grid(B * H, Dv / cols);
  tree_gdn_kernel<<<grid, cols * kQ, 0, static_cast<cudaStream_t>(stream)>>>(
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
  if (Dk != kDk || Dv <= 0 || Dv % 32 || (Dv > kColsPerBlock && Dv % kColsPerBlock)) return CFB_ERR_UNSUPPORTED;
  const unsigned long long need = (unsigned long long)B * N * H * Dk * Dv;
  if (need > (unsigned long long)CFB_TREE_GDN_NOALLOC_MAX_FLOATS) return CFB_ERR_WORKSPACE;
  float* scratch = nullptr;
  const cfb_status st = scratch_for_current_device(&scratch);
  if (st != CFB_OK) return st;
  const int cols = Dv < kColsPerBlock ? Dv : kColsPerBlock;
  const dim3 grid(B * H, Dv / cols);
  tree_gdn_kernel<<<grid, cols * kQ, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const __half*>(q), static_cast<const __half*>(k), static_cast<const __half*>(v), g, beta,
      parent, init, o, scratch, N, H, Dv, use_l2norm);
  return cfb_launch_status("tree_gdn_kernel (no-alloc)");
}
