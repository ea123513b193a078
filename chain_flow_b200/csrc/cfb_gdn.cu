// cfb_gdn.cu -- tree-aware Gated-DeltaNet verification (sm_100a).
//
// Restates the recurrence of the reference's tree scan (src/chain_flow/kernels/tree_scan.py:29-78)
// and the fork's verify kernels (patch tree_gdn.py:3285-3385, tree_gdn_verify.cu:4401-4562).
// Per node n with parent p (p < 0: the shared prefix state):
//     S = S_p * exp(g_n);  S += k_n (x) beta_n (v_n - S^T k_n);  o_n = S^T q_n
// q, k are L2-normalised as x / (||x|| + 1e-6) and q is scaled by Dk**-0.5 (tree_scan.py:25-27).
//
// cfb_tree_gdn runs it node by node (tree_gdn_kernel: nodes arrive in BFS order, parent < child,
// so walking them in index order finds every parent state already written; one CTA per request,
// head and 32 value columns, a warp per quarter of the Dk = 128 key rows, a lane per value
// column), or, for launches too small to fill the GPU that way, path-parallel
// (tree_gdn_path_kernel: one CTA per node, head and 32 value columns, walking the node's ancestor
// chain from the prefix state with the same per-node arithmetic). cfb_tree_gdn_verify is the
// in-engine verify (gate from A_log / dt_bias / a / b, state slots, ancestor chains), and
// cfb_tree_gdn_factor its shared-root factorisation.
#include <cuda_runtime.h>
#include <cuda_fp16.h>
#include <cuda_bf16.h>
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
// cfb_tree_gdn runs path-parallel (tree_gdn_path_kernel) when the node-by-node grid has fewer
// (request, head, column block) CTAs than the device has SMs. Measured at 16 heads, Dv = 128
// (64 CTAs a request): 1 request 13.1 against 19.9 us, 2 requests 19.3 against 20.5 us, 3 requests
// 27.6 against 26.9 us (path-parallel against node by node).
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
    // a parent must be -1 (the prefix state) or an earlier node of the same tree; any other
    // value is never dereferenced: the node (and every descendant) gets NaN state and output
    const bool bad = p >= n || p < -1;
    if ((p != held || bad) && live) {
      if (bad) {
#pragma unroll
        for (int i = 0; i < kRowsPerThread; ++i) S[i] = __int_as_float(0x7fc00000);
      } else {
        const float* src = (p < 0) ? init + ((size_t)b * H + h) * kDk * Dv
                                   : states + (((size_t)b * N + p) * H + h) * kDk * Dv;
#pragma unroll
        for (int i = 0; i < kRowsPerThread; ++i) S[i] = src[(size_t)(k0 + i) * Dv + j];
      }
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

// The same recurrence, path-parallel, for launches too small to fill the GPU node by node: one CTA
// per (request, node, head, 32 value columns), with tree_gdn_kernel's thread layout. The CTA
// issues its prefix-state loads first, finds its node's ancestor chain in the tree's parent array,
// stages only the chain's keys (fp32, with their L2 norms, g and beta) and its own node's query,
// and walks the chain with the state in registers, node by node with tree_gdn_kernel's arithmetic
// (the same operations in the same order). It writes only its own node's state and output, so no
// state is re-read; ancestors are recomputed instead (about depth + 1 node steps a node). A
// parent that is neither -1 nor an earlier node of the tree gives NaN on every node below it, as
// in tree_gdn_kernel; the bad index is never dereferenced.
inline size_t gdn_path_smem(int N) { return (size_t)(N + 1) * kDk * 4 + (size_t)N * (5 * 4 + kColsPerBlock * 4); }

__global__ void __launch_bounds__(kColsPerBlock * kQ, kMinBlocks)
tree_gdn_path_kernel(const __half* __restrict__ q, const __half* __restrict__ k, const __half* __restrict__ v,
                     const float* __restrict__ g, const float* __restrict__ beta, const int32_t* __restrict__ parent,
                     const float* __restrict__ init, float* __restrict__ o, float* __restrict__ states, int N,
                     int H, int Dv, int use_l2norm) {
  extern __shared__ float gsm[];
  float (*ks)[kDk] = reinterpret_cast<float (*)[kDk]>(gsm);           // [N] chain keys, root first
  float* qs = gsm + (size_t)N * kDk;                                  // [kDk] the node's query
  float* nk = qs + kDk;                                               // [N] key norms
  float* gd = nk + N;                                                 // [N] exp(g)
  float* bt = gd + N;                                                 // [N] beta
  int* ch = reinterpret_cast<int*>(bt + N);                           // [N] chain node ids, root first
  float (*vs)[kColsPerBlock] = reinterpret_cast<float (*)[kColsPerBlock]>(ch + N);   // [N] v of the columns
  __shared__ float red[2][2][kQ][kColsPerBlock];
  __shared__ int s_nd, s_bad;
  __shared__ float s_nq;
  const int bn = blockIdx.x;
  const int b = bn / N, n = bn % N, h = blockIdx.y;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int j = blockIdx.z * kColsPerBlock + lane;     // value column
  const int k0 = warp * kRowsPerThread;
  const float scale = rsqrtf((float)kDk);
  const bool live = j < Dv;
  // the prefix state first: its loads are in flight while the chain is found and staged
  float S[kRowsPerThread];
  {
    const float* src = init + ((size_t)b * H + h) * kDk * Dv;
#pragma unroll
    for (int i = 0; i < kRowsPerThread; ++i) S[i] = live ? src[(size_t)(k0 + i) * Dv + j] : 0.f;
  }
  // the tree's parent array, one load a thread, then the chain walked in shared memory
  int* pr = reinterpret_cast<int*>(vs + N);                         // [N]
  for (int m = tid; m < N; m += blockDim.x) pr[m] = parent[(size_t)b * N + m];
  __syncthreads();
  if (tid == 0) {   // the chain, leaf first in ch, then reversed to root first
    int nd = 0, bad = 0;
    for (int c = n; c >= 0 && nd < N;) {
      ch[nd++] = c;
      const int p = pr[c];
      if (p >= c || p < -1) { bad = 1; break; }
      c = p;
    }
    for (int i = 0; i < nd / 2; ++i) { const int t = ch[i]; ch[i] = ch[nd - 1 - i]; ch[nd - 1 - i] = t; }
    s_nd = nd; s_bad = bad;
  }
  __syncthreads();
  const int nd = s_nd;
  // stage the chain's keys and the node's query (fp16 -> fp32), 16-byte loads all in flight
  for (int e = tid; e < (nd + 1) * (kDk / 8); e += blockDim.x) {
    const int r = e / (kDk / 8), c = e - r * (kDk / 8);
    const int m = r < nd ? ch[r] : n;
    const size_t nh = ((size_t)b * N + m) * H + h;
    const uint4 a = *reinterpret_cast<const uint4*>((r < nd ? k : q) + nh * kDk + c * 8);
    const __half2* a2 = reinterpret_cast<const __half2*>(&a);
    float* dst = r < nd ? ks[r] : qs;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float2 f = __half22float2(a2[i]);
      dst[c * 8 + 2 * i] = f.x; dst[c * 8 + 2 * i + 1] = f.y;
    }
  }
  for (int e = tid; e < nd * kColsPerBlock; e += blockDim.x) {
    const int r = e / kColsPerBlock, c = e - r * kColsPerBlock;
    const int col = blockIdx.z * kColsPerBlock + c;
    const size_t nh = ((size_t)b * N + ch[r]) * H + h;
    vs[r][c] = col < Dv ? __half2float(v[nh * Dv + col]) : 0.f;
  }
  for (int r = tid; r < nd; r += blockDim.x) {
    const size_t nh = ((size_t)b * N + ch[r]) * H + h;
    gd[r] = __expf(g[nh]);
    bt[r] = beta[nh];
  }
  __syncthreads();
  // L2 norms as tree_gdn_kernel takes them (one warp per row)
  for (int rr = warp; rr <= nd; rr += blockDim.x >> 5) {
    const float* src = rr < nd ? ks[rr] : qs;
    float ss = 0.f;
    for (int i = lane; i < kDk; i += 32) ss += src[i] * src[i];
    for (int off = 16; off > 0; off >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, off);
    if (lane == 0) {
      const float inv = use_l2norm ? 1.f / (sqrtf(ss) + 1e-6f) : 1.f;
      if (rr < nd) nk[rr] = inv; else s_nq = inv * scale;
    }
  }
  __syncthreads();
  if (s_bad) {
#pragma unroll
    for (int i = 0; i < kRowsPerThread; ++i) S[i] = __int_as_float(0x7fc00000);
  }
  for (int r = 0; r < nd; ++r) {
    const int par = r & 1;
    const float decay = gd[r], kn = nk[r];
    float kv = 0.f;
#pragma unroll
    for (int i = 0; i < kRowsPerThread; ++i) { S[i] *= decay; kv += S[i] * ks[r][k0 + i]; }
    red[par][0][warp][lane] = kv;
    __syncthreads();
    kv = (red[par][0][0][lane] + red[par][0][1][lane] + red[par][0][2][lane] + red[par][0][3][lane]) * kn;
    const float delta = (vs[r][lane] - kv) * bt[r];
#pragma unroll
    for (int i = 0; i < kRowsPerThread; ++i) S[i] += (ks[r][k0 + i] * kn) * delta;
  }
  float on = 0.f;
  const size_t nh = ((size_t)b * N + n) * H + h;
  float* dst = states + nh * kDk * Dv;
#pragma unroll
  for (int i = 0; i < kRowsPerThread; ++i) {
    on += S[i] * qs[k0 + i];
    if (live) __stcs(dst + (size_t)(k0 + i) * Dv + j, S[i]);
  }
  red[nd & 1][1][warp][lane] = on;
  __syncthreads();
  if (warp == 0 && live)
    o[nh * Dv + j] = (red[nd & 1][1][0][lane] + red[nd & 1][1][1][lane] + red[nd & 1][1][2][lane] +
                      red[nd & 1][1][3][lane]) * s_nq;
}

// the current device's SM count, looked up once per device
cfb_status device_sms(int* out) {
  static std::mutex mu;
  static int sms[128] = {};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return cfb_launch_status("cudaGetDevice");
  std::lock_guard<std::mutex> lock(mu);
  if (dev >= 0 && dev < 128 && sms[dev] > 0) { *out = sms[dev]; return CFB_OK; }
  int n = 0;
  if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0)
    return cfb_launch_status("cudaDeviceGetAttribute(multiprocessor count)");
  if (dev >= 0 && dev < 128) sms[dev] = n;
  *out = n;
  return CFB_OK;
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
  if (cudaFuncSetAttribute(tree_gdn_path_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           (int)gdn_path_smem(kMaxNodes)) != cudaSuccess)
    return cfb_launch_status("tree_gdn_path_kernel shared-memory attribute");
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
  // node by node while the (request, head, column block) CTAs fill the GPU; path-parallel below
  int sms = 0;
  if (device_sms(&sms) != CFB_OK) return CFB_ERR_CUDA;
  if ((long long)B * H * (Dv / kColsPerBlock) < sms) {
    const dim3 grid(B * N, H, Dv / kColsPerBlock);
    tree_gdn_path_kernel<<<grid, kColsPerBlock * kQ, gdn_path_smem(N), static_cast<cudaStream_t>(stream)>>>(
        static_cast<const __half*>(q), static_cast<const __half*>(k), static_cast<const __half*>(v), g, beta,
        parent, init, o, states, N, H, Dv, use_l2norm);
    return cfb_launch_status("tree_gdn_path_kernel");
  }
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

// =================================================================================================
// The in-engine tree GDN verify: the contract of the reference's vLLM-patch kernel
// (gdn_verify_kernel, src/chain_flow/patches/vllm-0.25.1-chain-flow-tree.patch:4401-4562). The gate
// comes from the model's raw parameters (decay exp(-exp(A_log) softplus(a + dt_bias)),
// beta = sigmoid(b)), states live in slots [slots, HV, V, K] (K = 128 contiguous), and every
// query row t re-walks its ancestor chain chain[t, depth[t]] .. chain[t, 0] from its initial
// slot, then writes its output row and its state to its own slot.
//
// One CTA per (query row, value head, kVRows value rows). Each value row's 128 keys are split over
// kRowParts = 8 lanes, and a lane holds kLaneRows = 2 rows: lane l = 8 g + c holds key chunks c,
// c + 8, c + 16, c + 24 (16 columns) of rows 2g and 2g + 1 of its warp's 8 rows. A warp's 16-byte
// access then covers 4 rows x 128 contiguous bytes, so every state load and store moves whole
// lines straight between global memory and registers. A row's S k (and S q) sum closes over its
// 8 lanes with 3 shuffles that leave row 2g + (l >> 2) % 2's total in lane l, and 2 indexed
// shuffles return the rows' updates. The per-node decay is a scalar shared by every element of
// the CTA, so the state is held as S = G U: a node's decay multiplies only G, and U takes the
// update divided by G (when G falls below kFoldBelow it is folded into U). The state loads are
// issued first; while they are in flight the CTA stages the ancestor chain (at most kMaxChain
// nodes) in shared memory: the chain row, then, all loads at once, each node's normalised key
// (fp32), decay and beta, the value of every row of the CTA, and the query.
namespace {

enum { GV_F32 = 0, GV_F16 = 1, GV_BF16 = 2 };
constexpr int kMaxChain = 16;              // nodes on one row's chain (tree depth + 1)
constexpr int kRowParts = 8;               // lanes sharing one value row's keys
constexpr int kLaneRows = 2;               // value rows a lane holds
constexpr int kWarpRows = 32 / kRowParts * kLaneRows;      // 8
constexpr int kLaneChunks = kDk / 4 / kRowParts;           // 16-byte key chunks of a row per lane
constexpr int kVerifyThreads = 128;
constexpr int kVerifyMinBlocks = 6;        // CTAs per SM the register budget is cut for
constexpr int kVRows = kVerifyThreads / 32 * kWarpRows;   // value rows per CTA
constexpr float kFoldBelow = 1e-20f;       // the decay product folded into the state below this

__device__ __forceinline__ float ld_code(const void* p, int code, long long i) {
  if (code == GV_F32) return static_cast<const float*>(p)[i];
  if (code == GV_F16) return __half2float(static_cast<const __half*>(p)[i]);
  return __bfloat162float(static_cast<const __nv_bfloat16*>(p)[i]);
}
__device__ __forceinline__ float to_f(__half x) { return __half2float(x); }
__device__ __forceinline__ float to_f(__nv_bfloat16 x) { return __bfloat162float(x); }
__device__ __forceinline__ void from_f(__half& d, float x) { d = __float2half_rn(x); }
__device__ __forceinline__ void from_f(__nv_bfloat16& d, float x) { d = __float2bfloat16_rn(x); }

struct VerifyArgs {
  const void* A_log; int c_alog;
  const void* dt_bias; int c_dtb;
  const void* a; int c_a;
  const void* b; int c_b;
  const void* q; const void* k; const void* v; void* o;
  float* state; long long slot_stride;
  const int* chain; int chain_stride;
  const int* depth; const int* out_slot; const int* init_slot; const int* rows;
  float scale, threshold;
  int H, HV, V, write_out, write_state;
};

// The sum over a row's 8 lanes of a[(lane >> 2) % 2]: lane bit 2 picks the row it keeps (adding
// its partner's copy of that row), then the sum runs over lane bits 1 and 0.
__device__ __forceinline__ float row_pair_sum(const float (&a)[kLaneRows], int lane) {
  const bool b2 = lane & 4;
  float d = (b2 ? a[1] : a[0]) + __shfl_xor_sync(0xffffffffu, b2 ? a[0] : a[1], 4);
  d += __shfl_xor_sync(0xffffffffu, d, 2);
  d += __shfl_xor_sync(0xffffffffu, d, 1);
  return d;
}

// (x . y) over a lane's chunks
__device__ __forceinline__ float chunk_dot(const float4 (&x)[kLaneChunks], const float4 (&y)[kLaneChunks]) {
  float p0 = 0.f, p1 = 0.f, p2 = 0.f, p3 = 0.f;
#pragma unroll
  for (int i = 0; i < kLaneChunks; ++i) {
    p0 += x[i].x * y[i].x; p1 += x[i].y * y[i].y; p2 += x[i].z * y[i].z; p3 += x[i].w * y[i].w;
  }
  return (p0 + p1) + (p2 + p3);
}

template <typename T>
__global__ void __launch_bounds__(kVerifyThreads, kVerifyMinBlocks) tree_gdn_verify_kernel(const VerifyArgs A) {
  __shared__ float4 ks[kMaxChain][kDk / 4];   // normalised keys, processing order (root first)
  __shared__ float vs[kMaxChain][kVRows];
  __shared__ float egs[kMaxChain], bts[kMaxChain];
  __shared__ float4 qs[kDk / 4];
  __shared__ int chs[kMaxChain];              // the row's chain: chs[0] is the row's own node
  const int tt = blockIdx.x, hv = blockIdx.y;
  const int vbase = blockIdx.z * kVRows;                  // the CTA's first value row
  const int t = A.rows ? A.rows[tt] : tt;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int row0 = vbase + warp * kWarpRows;              // the warp's first value row
  const int nlive = min(kWarpRows, A.V - row0);           // the warp's rows inside V
  const int h = hv / (A.HV / A.H);
  const T* q = static_cast<const T*>(A.q);
  const T* k = static_cast<const T*>(A.k);
  const T* v = static_cast<const T*>(A.v);
  const int g = lane >> 3, c = lane & (kRowParts - 1);    // row pair, part of the row
  const long long sbase = ((long long)hv * A.V + row0 + kLaneRows * g) * kDk;
  // one round trip for everything the later loads are addressed by: the row's slots, depth and
  // whole chain row (chain[t, depth] .. chain[t, 0] is the walk from the root end)
  const int islot = A.init_slot[t];
  const int oslot = A.write_state ? A.out_slot[t] : 0;
  // a depth that does not fit the chain row walks nothing and gives NaN (no entry past the row
  // is ever used as a node index)
  const int dep = A.depth[t];
  const bool bad_depth = dep < 0 || dep >= A.chain_stride;
  const int nd = bad_depth ? 0 : dep + 1;                // chain_stride <= kMaxChain
  const int chv = tid < A.chain_stride ? A.chain[(long long)t * A.chain_stride + tid] : 0;
  const float negA = -expf(ld_code(A.A_log, A.c_alog, hv));
  const float dtb = ld_code(A.dt_bias, A.c_dtb, hv);
  // the lane's chunks of its two state rows, in flight while the chain is staged
  float4 S[kLaneRows][kLaneChunks];
  {
    const float4* src = reinterpret_cast<const float4*>(A.state + (long long)islot * A.slot_stride + sbase) + c;
#pragma unroll
    for (int rr = 0; rr < kLaneRows; ++rr)
#pragma unroll
      for (int i = 0; i < kLaneChunks; ++i)
        S[rr][i] = kLaneRows * g + rr < nlive ? __ldcg(src + rr * (kDk / 4) + kRowParts * i) : make_float4(0.f, 0.f, 0.f, 0.f);
  }
  if (bad_depth) {
#pragma unroll
    for (int rr = 0; rr < kLaneRows; ++rr)
#pragma unroll
      for (int i = 0; i < kLaneChunks; ++i) {
        const float nan = __int_as_float(0x7fc00000);
        S[rr][i] = make_float4(nan, nan, nan, nan);
      }
  }
  if (tid < A.chain_stride) chs[tid] = chv;
  constexpr int kWarps = kVerifyThreads / 32;
  __syncthreads();
  // warp w takes nodes j = w, w + kWarps, ...; lane l holds key columns 4l .. 4l+3
  for (int j = warp; j < nd; j += kWarps) {
    const int n = chs[nd - 1 - j];
    const T* kr = k + ((long long)n * A.H + h) * kDk + lane * 4;
    const float k0 = to_f(kr[0]), k1 = to_f(kr[1]), k2 = to_f(kr[2]), k3 = to_f(kr[3]);
    float ss = (k0 * k0 + k1 * k1) + (k2 * k2 + k3 * k3);
    for (int off = 16; off > 0; off >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, off);
    const float inv = rsqrtf(ss + 1e-6f);
    ks[j][lane] = make_float4(k0 * inv, k1 * inv, k2 * inv, k3 * inv);
    if (lane == 0) {
      const float x = ld_code(A.a, A.c_a, (long long)n * A.HV + hv) + dtb;
      const float sp = x <= A.threshold ? log1pf(expf(x)) : x;
      egs[j] = expf(negA * sp);
      bts[j] = 1.f / (1.f + expf(-ld_code(A.b, A.c_b, (long long)n * A.HV + hv)));
    }
  }
  {   // every (chain node, value row) of the CTA: element e = j * kVRows + row, all loads first
    constexpr int kPer = (kMaxChain * kVRows + kVerifyThreads - 1) / kVerifyThreads;
    T vv[kPer];
#pragma unroll
    for (int i = 0; i < kPer; ++i) {
      const int e = tid + kVerifyThreads * i, j = e / kVRows, vr = vbase + e % kVRows;
      if (j < nd && vr < A.V) vv[i] = v[((long long)chs[nd - 1 - j] * A.HV + hv) * A.V + vr];
    }
#pragma unroll
    for (int i = 0; i < kPer; ++i) {
      const int e = tid + kVerifyThreads * i, j = e / kVRows, vr = vbase + e % kVRows;
      if (j < nd) vs[j][e % kVRows] = vr < A.V ? to_f(vv[i]) : 0.f;
    }
  }
  if (A.write_out && warp == kWarps - 1) {
    const T* qr = q + ((long long)t * A.H + h) * kDk + lane * 4;
    const float q0 = to_f(qr[0]), q1 = to_f(qr[1]), q2 = to_f(qr[2]), q3 = to_f(qr[3]);
    float ss = (q0 * q0 + q1 * q1) + (q2 * q2 + q3 * q3);
    for (int off = 16; off > 0; off >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, off);
    const float inv = rsqrtf(ss + 1e-6f) * A.scale;
    qs[lane] = make_float4(q0 * inv, q1 * inv, q2 * inv, q3 * inv);
  }
  __syncthreads();
  const int myrow = kLaneRows * g + ((lane >> 2) & 1);   // the row whose sums this lane receives
  // the walk: S <- S exp(g); S += beta (v - S k) k^T, node by node from the root end, on S = G U
  float G = 1.f;
  for (int j = 0; j < nd; ++j) {
    float Gj = G * egs[j];
    if (Gj < kFoldBelow) {       // the same for every thread of the CTA
#pragma unroll
      for (int rr = 0; rr < kLaneRows; ++rr)
#pragma unroll
        for (int i = 0; i < kLaneChunks; ++i) { S[rr][i].x *= Gj; S[rr][i].y *= Gj; S[rr][i].z *= Gj; S[rr][i].w *= Gj; }
      Gj = 1.f;
    }
    float4 kk[kLaneChunks];
#pragma unroll
    for (int i = 0; i < kLaneChunks; ++i) kk[i] = ks[j][c + kRowParts * i];
    float a[kLaneRows];
#pragma unroll
    for (int rr = 0; rr < kLaneRows; ++rr) a[rr] = chunk_dot(S[rr], kk);
    const float p = Gj * row_pair_sum(a, lane);
    const float dm = (vs[j][warp * kWarpRows + myrow] - p) * bts[j] / Gj;
    float d[kLaneRows];
#pragma unroll
    for (int rr = 0; rr < kLaneRows; ++rr) d[rr] = __shfl_sync(0xffffffffu, dm, kRowParts * g + 4 * rr);
#pragma unroll
    for (int rr = 0; rr < kLaneRows; ++rr)
#pragma unroll
      for (int i = 0; i < kLaneChunks; ++i) {
        S[rr][i].x += d[rr] * kk[i].x; S[rr][i].y += d[rr] * kk[i].y;
        S[rr][i].z += d[rr] * kk[i].z; S[rr][i].w += d[rr] * kk[i].w;
      }
    G = Gj;
  }
  if (A.write_out) {
    float4 qq[kLaneChunks];
#pragma unroll
    for (int i = 0; i < kLaneChunks; ++i) qq[i] = qs[c + kRowParts * i];
    float a[kLaneRows];
#pragma unroll
    for (int rr = 0; rr < kLaneRows; ++rr) a[rr] = chunk_dot(S[rr], qq);
    const float o = G * row_pair_sum(a, lane);
    if ((lane & 3) == 0 && myrow < nlive)
      from_f(static_cast<T*>(A.o)[((long long)t * A.HV + hv) * A.V + row0 + myrow], o);
  }
  if (A.write_state) {
    float4* dst = reinterpret_cast<float4*>(A.state + (long long)oslot * A.slot_stride + sbase) + c;
#pragma unroll
    for (int rr = 0; rr < kLaneRows; ++rr)
      if (kLaneRows * g + rr < nlive) {
#pragma unroll
        for (int i = 0; i < kLaneChunks; ++i)
          dst[rr * (kDk / 4) + kRowParts * i] = make_float4(G * S[rr][i].x, G * S[rr][i].y, G * S[rr][i].z, G * S[rr][i].w);
      }
  }
}

}  // namespace

extern "C" cfb_status cfb_tree_gdn_verify(const void* A_log, int A_log_dtype, const void* dt_bias, int dt_bias_dtype,
                                          const void* a, int a_dtype, const void* b, int b_dtype, const void* q,
                                          const void* k, const void* v, void* o, int qkv_dtype, float* state,
                                          int64_t slot_stride, const int32_t* chain, int chain_stride,
                                          const int32_t* depth, const int32_t* out_slot, const int32_t* init_slot,
                                          const int32_t* rows, float scale, int T_rows, int H, int HV, int K, int V,
                                          int write_out, int write_state, void* stream) {
  if (!A_log || !dt_bias || !a || !b || !q || !k || !v || !state || !chain || !depth || !out_slot || !init_slot ||
      (write_out && !o) || T_rows < 0 || H <= 0 || HV <= 0 || chain_stride <= 0)
    return CFB_ERR_INVALID_ARG;
  for (int c : {A_log_dtype, dt_bias_dtype, a_dtype, b_dtype})
    if (c < GV_F32 || c > GV_BF16) return CFB_ERR_INVALID_ARG;
  if (K != kDk || V <= 0 || V % 32 || HV % H || chain_stride > kMaxChain ||
      (qkv_dtype != GV_F16 && qkv_dtype != GV_BF16))
    return CFB_ERR_UNSUPPORTED;
  if ((reinterpret_cast<uintptr_t>(state) & 15) || slot_stride < (int64_t)HV * V * K || slot_stride % 4)
    return CFB_ERR_INVALID_ARG;
  if (T_rows == 0) return CFB_OK;
  VerifyArgs A{A_log, A_log_dtype, dt_bias, dt_bias_dtype, a, a_dtype, b, b_dtype, q, k, v, o, state,
               slot_stride, chain, chain_stride, depth, out_slot, init_slot, rows, scale, 20.0f,
               H, HV, V, write_out, write_state};
  const dim3 grid((unsigned)T_rows, (unsigned)HV, (unsigned)((V + kVRows - 1) / kVRows));
  if (qkv_dtype == GV_F16)
    tree_gdn_verify_kernel<__half><<<grid, kVerifyThreads, 0, static_cast<cudaStream_t>(stream)>>>(A);
  else
    tree_gdn_verify_kernel<__nv_bfloat16><<<grid, kVerifyThreads, 0, static_cast<cudaStream_t>(stream)>>>(A);
  return cfb_launch_status("tree_gdn_verify_kernel");
}

// =================================================================================================
// Shared-root factorisation of the tree GDN verify (the contract of the reference fork's
// gdn_factor, src/chain_flow/patches/vllm-0.25.1-chain-flow-tree.patch:4664-5094): the outputs of
// every row of a request whose rows all start from ONE state slot H, with no per-node state read
// or written. Every update along a path is rank 1, so (k^ = k * rsqrt(|k|^2 + 1e-6),
// q^ = q * rsqrt(|q|^2 + 1e-6) * scale, g the decay, beta the gate)
//   h_t = D_t H + sum_{m on t's path} w_{m,t} u_m k^_m^T,  D_t = g_t D_p,  w_{m,t} = g_t w_{m,p},
//   w_{t,t} = 1,  u_t = beta_t (v_t - g_t S_t),
//   S_t = h_p k^_t = D_p (H k^_t) + sum_{m on p's path} w_{m,p} (k^_m . k^_t) u_m,
//   o_t = h_t q^_t = D_t (H q^_t) + sum_{m on t's path} w_{m,t} (k^_m . q^_t) u_m.
// H is touched only through the matrix-vector products H k^_t and H q^_t; the rest is dot products
// of the small k / q vectors and a level-by-level solve for the u_t.
//
// One CTA per (32 value rows, value head, request), 8 warps. The CTA stages the request's
// normalised keys and queries, gates, values and chains, and its 32 rows of H (padded rows in
// shared memory, then each warp holds them in registers, one row per lane); warp w forms the
// products H k^_j / H q^_j for j = w, w + 8, ... with the vectors broadcast from shared memory.
// The ancestor dot products take a warp each. Then the nodes are solved level by level (a warp per
// node, a lane per value row) and every node's output is contracted.
namespace {

constexpr int kFacWarps = 8;
constexpr int kFacThreads = kFacWarps * 32;
constexpr int kFacBV = 32;                 // value rows per CTA
constexpr int kFacMaxN = 64;               // rows per request
constexpr int kFacMaxW = kMaxChain;        // chain entries per row (depth + 1)
constexpr int kFacHLd = kDk + 4;           // padded row of the staged H block

struct FactorArgs {
  const void* A_log; int c_alog;
  const void* dt_bias; int c_dtb;
  const void* a; int c_a;
  const void* b; int c_b;
  const void* q; const void* k; const void* v; void* o;
  const float* state; long long slot_stride;
  const int* chain; int chain_stride;
  const int* depth; const int* init_slot; const int* row_start; const int* row_count;
  float scale, threshold;
  int H, HV, V, n_max;
};

// shared memory of one CTA for requests of up to n rows (floats, then ints)
inline size_t factor_smem(int n) {
  const size_t f = (size_t)2 * n * kDk            // k^, q^
                   + (size_t)kFacBV * kFacHLd      // H block
                   + (size_t)4 * n * kFacBV        // H k^, H q^, u, v
                   + (size_t)3 * n                 // g, beta, D
                   + (size_t)3 * n * kFacMaxW;     // w, (k^_m . k^_t), (k^_m . q^_t)
  const size_t i = (size_t)n * kFacMaxW + 3 * (size_t)n + kFacMaxW;   // chains, depths, levels, flags
  return (f + i) * 4;
}

template <typename T>
__global__ void __launch_bounds__(kFacThreads) tree_gdn_factor_kernel(const FactorArgs A) {
  extern __shared__ __align__(16) float fsm[];
  const int vb = blockIdx.x, hv = blockIdx.y, s = blockIdx.z;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int h = hv / (A.HV / A.H);
  const int base = A.row_start[s], n = A.row_count[s];
  const int NM = A.n_max;
  float* xk = fsm;                                   // [NM][kDk]
  float* xq = xk + (size_t)NM * kDk;                 // [NM][kDk]
  float* sH = xq + (size_t)NM * kDk;                 // [kFacBV][kFacHLd]
  float* sP = sH + (size_t)kFacBV * kFacHLd;         // [NM][kFacBV]  H k^
  float* sQ = sP + (size_t)NM * kFacBV;              //               H q^
  float* sU = sQ + (size_t)NM * kFacBV;
  float* sV = sU + (size_t)NM * kFacBV;
  float* sg = sV + (size_t)NM * kFacBV;
  float* sb = sg + NM;
  float* sD = sb + NM;
  float* sW = sD + NM;                               // [NM][kFacMaxW]
  float* sC = sW + (size_t)NM * kFacMaxW;            // C[t][j] = k^_{m_j} . k^_t
  float* sR = sC + (size_t)NM * kFacMaxW;            // R[t][j] = k^_{m_j} . q^_t
  int* sCh = reinterpret_cast<int*>(sR + (size_t)NM * kFacMaxW);   // [NM][kFacMaxW] local ids
  int* sDep = sCh + (size_t)NM * kFacMaxW;
  int* sLev = sDep + NM;                             // nodes sorted by depth
  int* sLevN = sLev + NM;                            // [kFacMaxW] first index of each depth
  int* sbad = sLevN + kFacMaxW;                      // [NM] rows with an unusable chain
  if (n <= 0) return;
  const T* q = static_cast<const T*>(A.q);
  const T* k = static_cast<const T*>(A.k);
  const T* v = static_cast<const T*>(A.v);
  const int v0 = vb * kFacBV;
  // chains (local ids), depths, gates, values, and the H block
  for (int t = tid; t < n; t += kFacThreads) {
    // a depth past the chain row, or a chain entry outside this request's rows, is never used
    // as an index: the row is computed as a root-level node and its output is NaN
    const int dep = A.depth[base + t];
    bool bad = dep < 0 || dep >= A.chain_stride;
    const int d = bad ? 0 : dep;
    for (int j = 0; j <= d; ++j) {
      const int m = A.chain[(long long)(base + t) * A.chain_stride + j] - base;
      const bool ok = m >= 0 && m < n && (j > 0 || m == t);
      bad |= !ok;
      sCh[t * kFacMaxW + j] = ok ? m : t;
    }
    sDep[t] = bad ? 0 : d;
    sbad[t] = bad;
    const float x = ld_code(A.a, A.c_a, (long long)(base + t) * A.HV + hv) + ld_code(A.dt_bias, A.c_dtb, hv);
    const float sp = x <= A.threshold ? log1pf(expf(x)) : x;
    sg[t] = expf(-expf(ld_code(A.A_log, A.c_alog, hv)) * sp);
    sb[t] = 1.f / (1.f + expf(-ld_code(A.b, A.c_b, (long long)(base + t) * A.HV + hv)));
  }
  for (int e = tid; e < n * kFacBV; e += kFacThreads) {
    const int t = e / kFacBV, vl = e - t * kFacBV;
    sV[t * kFacBV + vl] = to_f(v[((long long)(base + t) * A.HV + hv) * A.V + v0 + vl]);
  }
  {
    const float4* src = reinterpret_cast<const float4*>(
        A.state + (long long)A.init_slot[base] * A.slot_stride + ((long long)hv * A.V + v0) * kDk);
    for (int e = tid; e < kFacBV * (kDk / 4); e += kFacThreads) {
      const int r = e / (kDk / 4), c4 = e - r * (kDk / 4);
      *reinterpret_cast<float4*>(&sH[r * kFacHLd + 4 * c4]) = src[e];
    }
  }
  // normalised keys and queries: a warp per row, lane l holds columns 4l .. 4l+3
  for (int rr = warp; rr < 2 * n; rr += kFacWarps) {
    const bool isq = rr >= n;
    const int t = isq ? rr - n : rr;
    const T* src = (isq ? q : k) + ((long long)(base + t) * A.H + h) * kDk + lane * 4;
    const float e0 = to_f(src[0]), e1 = to_f(src[1]), e2 = to_f(src[2]), e3 = to_f(src[3]);
    float ss = (e0 * e0 + e1 * e1) + (e2 * e2 + e3 * e3);
    for (int off = 16; off > 0; off >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, off);
    const float inv = rsqrtf(ss + 1e-6f) * (isq ? A.scale : 1.f);
    *reinterpret_cast<float4*>((isq ? xq : xk) + (size_t)t * kDk + lane * 4) =
        make_float4(e0 * inv, e1 * inv, e2 * inv, e3 * inv);
  }
  __syncthreads();
  if (tid == 0) {                                    // level lists: nodes ordered by depth
    int cnt[kFacMaxW] = {};
    for (int t = 0; t < n; ++t) ++cnt[sDep[t]];
    int acc = 0;
    for (int d = 0; d < kFacMaxW; ++d) { sLevN[d] = acc; acc += cnt[d]; cnt[d] = sLevN[d]; }
    for (int t = 0; t < n; ++t) sLev[cnt[sDep[t]]++] = t;
  }
  // H k^_j and H q^_j: lane = value row, the row in registers
  {
    float hr[kDk];
#pragma unroll
    for (int c = 0; c < kDk / 4; ++c) {
      const float4 f = *reinterpret_cast<const float4*>(&sH[lane * kFacHLd + 4 * c]);
      hr[4 * c] = f.x; hr[4 * c + 1] = f.y; hr[4 * c + 2] = f.z; hr[4 * c + 3] = f.w;
    }
    for (int j = warp; j < 2 * n; j += kFacWarps) {
      const float* x = j < n ? xk + (size_t)j * kDk : xq + (size_t)(j - n) * kDk;
      float p0 = 0.f, p1 = 0.f, p2 = 0.f, p3 = 0.f;
#pragma unroll
      for (int c = 0; c < kDk / 4; ++c) {
        const float4 xx = *reinterpret_cast<const float4*>(x + 4 * c);
        p0 = fmaf(hr[4 * c], xx.x, p0); p1 = fmaf(hr[4 * c + 1], xx.y, p1);
        p2 = fmaf(hr[4 * c + 2], xx.z, p2); p3 = fmaf(hr[4 * c + 3], xx.w, p3);
      }
      (j < n ? sP : sQ)[(size_t)(j < n ? j : j - n) * kFacBV + lane] = (p0 + p1) + (p2 + p3);
    }
  }
  // the ancestor dot products: pair (t, j) -> C[t][j] (j >= 1) and R[t][j] (j >= 0)
  for (int t = warp; t < n; t += kFacWarps) {
    const float4 kt = *reinterpret_cast<const float4*>(xk + (size_t)t * kDk + lane * 4);
    const float4 qt = *reinterpret_cast<const float4*>(xq + (size_t)t * kDk + lane * 4);
    for (int j = 0; j <= sDep[t]; ++j) {
      const int m = sCh[t * kFacMaxW + j];
      const float4 km = *reinterpret_cast<const float4*>(xk + (size_t)m * kDk + lane * 4);
      float c = (km.x * kt.x + km.y * kt.y) + (km.z * kt.z + km.w * kt.w);
      float r = (km.x * qt.x + km.y * qt.y) + (km.z * qt.z + km.w * qt.w);
      for (int off = 16; off > 0; off >>= 1) {
        c += __shfl_xor_sync(0xffffffffu, c, off);
        r += __shfl_xor_sync(0xffffffffu, r, off);
      }
      if (lane == 0) { sC[t * kFacMaxW + j] = c; sR[t * kFacMaxW + j] = r; }
    }
  }
  __syncthreads();
  // level by level: u_t, D_t and the path weights w_{m,t}
  for (int d = 0; d < kFacMaxW; ++d) {
    const int l0 = sLevN[d], l1 = d + 1 < kFacMaxW ? sLevN[d + 1] : n;
    if (l0 >= l1) continue;
    for (int i = l0 + warp; i < l1; i += kFacWarps) {
      const int t = sLev[i];
      const int par = d > 0 ? sCh[t * kFacMaxW + 1] : -1;
      const float Dp = d > 0 ? sD[par] : 1.f;
      float S = Dp * sP[t * kFacBV + lane];
      for (int j = 1; j <= d; ++j) {
        const int m = sCh[t * kFacMaxW + j];
        S = fmaf(sW[par * kFacMaxW + j - 1] * sC[t * kFacMaxW + j], sU[m * kFacBV + lane], S);
      }
      const float g = sg[t];
      sU[t * kFacBV + lane] = sb[t] * (sV[t * kFacBV + lane] - g * S);
      if (lane <= d) sW[t * kFacMaxW + lane] = lane == 0 ? 1.f : sW[par * kFacMaxW + lane - 1] * g;
      if (lane == 0) sD[t] = Dp * g;
    }
    __syncthreads();
  }
  // outputs
  for (int t = warp; t < n; t += kFacWarps) {
    const int d = sDep[t];
    float acc = sD[t] * sQ[t * kFacBV + lane];
    for (int j = 0; j <= d; ++j) {
      const int m = sCh[t * kFacMaxW + j];
      acc = fmaf(sW[t * kFacMaxW + j] * sR[t * kFacMaxW + j], sU[m * kFacBV + lane], acc);
    }
    from_f(static_cast<T*>(A.o)[((long long)(base + t) * A.HV + hv) * A.V + v0 + lane],
           sbad[t] ? __int_as_float(0x7fc00000) : acc);
  }
}

cfb_status factor_smem_attr(size_t bytes) {
  static std::mutex mu;
  static size_t done[kMaxDevices] = {};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return cfb_launch_status("cudaGetDevice");
  if (dev < 0 || dev >= kMaxDevices) return CFB_ERR_UNSUPPORTED;
  std::lock_guard<std::mutex> lock(mu);
  if (done[dev] >= bytes) return CFB_OK;
  if (cudaFuncSetAttribute(tree_gdn_factor_kernel<__half>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes) !=
          cudaSuccess ||
      cudaFuncSetAttribute(tree_gdn_factor_kernel<__nv_bfloat16>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           (int)bytes) != cudaSuccess)
    return cfb_launch_status("tree_gdn_factor_kernel shared-memory attribute");
  done[dev] = bytes;
  return CFB_OK;
}

}  // namespace

extern "C" cfb_status cfb_tree_gdn_factor(const void* A_log, int A_log_dtype, const void* dt_bias, int dt_bias_dtype,
                                          const void* a, int a_dtype, const void* b, int b_dtype, const void* q,
                                          const void* k, const void* v, void* o, int qkv_dtype, const float* state,
                                          int64_t slot_stride, const int32_t* chain, int chain_stride,
                                          const int32_t* depth, const int32_t* init_slot, const int32_t* row_start,
                                          const int32_t* row_count, int S, int n_max, float scale, int H, int HV,
                                          int K, int V, void* stream) {
  if (!A_log || !dt_bias || !a || !b || !q || !k || !v || !o || !state || !chain || !depth || !init_slot ||
      !row_start || !row_count || S < 0 || H <= 0 || HV <= 0 || chain_stride <= 0 || n_max <= 0)
    return CFB_ERR_INVALID_ARG;
  for (int c : {A_log_dtype, dt_bias_dtype, a_dtype, b_dtype})
    if (c < GV_F32 || c > GV_BF16) return CFB_ERR_INVALID_ARG;
  if (K != kDk || V <= 0 || V % kFacBV || HV % H || n_max > kFacMaxN || chain_stride > kFacMaxW ||
      (qkv_dtype != GV_F16 && qkv_dtype != GV_BF16))
    return CFB_ERR_UNSUPPORTED;
  if ((reinterpret_cast<uintptr_t>(state) & 15) || slot_stride < (int64_t)HV * V * K || slot_stride % 4)
    return CFB_ERR_INVALID_ARG;
  if (S == 0) return CFB_OK;
  const size_t smem = factor_smem(n_max);
  const cfb_status sa = factor_smem_attr(smem);
  if (sa != CFB_OK) return sa;
  FactorArgs A{A_log, A_log_dtype, dt_bias, dt_bias_dtype, a, a_dtype, b, b_dtype, q, k, v, o, state, slot_stride,
               chain, chain_stride, depth, init_slot, row_start, row_count, scale, 20.0f, H, HV, V, n_max};
  const dim3 grid((unsigned)(V / kFacBV), (unsigned)HV, (unsigned)S);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (qkv_dtype == GV_F16) tree_gdn_factor_kernel<__half><<<grid, kFacThreads, smem, st>>>(A);
  else tree_gdn_factor_kernel<__nv_bfloat16><<<grid, kFacThreads, smem, st>>>(A);
  return cfb_launch_status("tree_gdn_factor_kernel");
}
