// cfb_ring.cu -- the per-request context ring of the proposer: the window of the last C target
// hidden states each request's draft is conditioned on (reference FlowDrafterProposer._init_ring /
// _ring_write / _ring_gather, src/chain_flow/vllm_plugin/flow_proposer.py:881-961).
//
// ring fp16 [slots, C + 1, H]: slot r holds request r's last C hidden states in circular order;
// row C is a trash row that masked-off writes go to. rpos[r] is the next write position,
// nval[r] <= C the number of valid rows. Both kernels only move fp16 rows (bit-exact), one CTA
// per request, 16-byte copies when H is a multiple of 8.
#include <cuda_runtime.h>
#include "cfb_common.cuh"

namespace {

constexpr int kRingThreads = 256, kRingMaxRows = 64;

// Copy nrows rows of H halves, row i from src[i] to dst[i] (row pointers in shared memory), all
// rows' chunks spread over the CTA with 4 loads in flight per thread before their stores.
__device__ __forceinline__ void copy_rows(__half* const* dst, const __half* const* src, int nrows, int H) {
  if ((H & 7) == 0) {
    const int cpr = H / 8, total = nrows * cpr;
    for (int i0 = threadIdx.x; i0 < total; i0 += 4 * blockDim.x) {
      uint4 v[4];
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const int i = i0 + u * blockDim.x;
        if (i < total) v[u] = *reinterpret_cast<const uint4*>(src[i / cpr] + (i % cpr) * 8);
      }
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const int i = i0 + u * blockDim.x;
        if (i < total) *reinterpret_cast<uint4*>(dst[i / cpr] + (i % cpr) * 8) = v[u];
      }
    }
  } else {
    for (int i = threadIdx.x; i < nrows * H; i += blockDim.x) dst[i / H][i % H] = src[i / H][i % H];
  }
}

__global__ void __launch_bounds__(kRingThreads) ring_write_kernel(__half* ring, int64_t* rpos, int64_t* nval, int C, int H,
                                                         const __half* sh, long long nsh, const int64_t* rows,
                                                         const int64_t* starts, const int64_t* cnt,
                                                         const uint8_t* wmask, const int64_t* path,
                                                         long long path_ld, int kmax) {
  __shared__ __half* dst[kRingMaxRows];
  __shared__ const __half* src[kRingMaxRows];
  const int b = blockIdx.x;
  const long long r = rows[b];
  const long long head = rpos[r];
  const long long n = cnt[b];
  const bool on = wmask[b] != 0;
  for (int j = threadIdx.x; j < kmax; j += blockDim.x) {
    const long long off = path ? (j == 0 ? 0 : 1 + path[r * path_ld + j - 1]) : j;
    const bool valid = j < n && on;
    long long s = 0;
    if (valid) s = min(max(starts[b] + off, 0ll), nsh - 1);
    const long long d = valid ? (head + j) % C : C;
    dst[j] = ring + (r * (C + 1) + d) * H;
    src[j] = sh + s * H;
  }
  __syncthreads();                                       // every thread has read rpos / nval
  copy_rows(dst, src, kmax, H);
  if (threadIdx.x == 0) {
    const long long add = on ? n : 0;
    rpos[r] = (head + add) % C;
    nval[r] = min(nval[r] + add, (long long)C);
  }
}

__global__ void __launch_bounds__(kRingThreads) ring_gather_kernel(const __half* ring, const int64_t* rpos,
                                                          const int64_t* nval, int C, int H, const int64_t* rows,
                                                          __half* out) {
  __shared__ __half* dst[kRingMaxRows];
  __shared__ const __half* src[kRingMaxRows];
  const int b = blockIdx.x;
  const long long r = rows[b];
  const long long m = nval[r], head = rpos[r];
  for (int j = threadIdx.x; j < C; j += blockDim.x) {
    const long long t = min(max((long long)j - (C - m), 0ll), max(m - 1, 0ll));
    const long long phys = (((head - m + t) % C) + C) % C;
    dst[j] = out + ((long long)b * C + j) * H;
    src[j] = ring + (r * (C + 1) + phys) * H;
  }
  __syncthreads();
  copy_rows(dst, src, C, H);
}

}  // namespace

extern "C" cfb_status cfb_ring_write(void* ring, int64_t* rpos, int64_t* nval, int slots, int C, int H,
                                     const void* sh, int64_t nsh, const int64_t* rows, const int64_t* starts,
                                     const int64_t* cnt, const uint8_t* wmask, const int64_t* path,
                                     int64_t path_ld, int B, int kmax, void* stream) {
  if (!ring || !rpos || !nval || !sh || !rows || !starts || !cnt || !wmask || slots <= 0 || C <= 0 || H <= 0 ||
      nsh <= 0 || B < 0 || kmax <= 0 || (path && path_ld < kmax - 1))
    return CFB_ERR_INVALID_ARG;
  if (kmax > kRingMaxRows || C > kRingMaxRows) return CFB_ERR_UNSUPPORTED;
  if ((H & 7) == 0 && ((reinterpret_cast<uintptr_t>(ring) | reinterpret_cast<uintptr_t>(sh)) & 15))
    return CFB_ERR_INVALID_ARG;
  if (B == 0) return CFB_OK;
  ring_write_kernel<<<B, kRingThreads, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<__half*>(ring), rpos, nval, C, H, static_cast<const __half*>(sh), nsh, rows, starts, cnt, wmask,
      path, path_ld, kmax);
  return cfb_launch_status("ring_write_kernel");
}

extern "C" cfb_status cfb_ring_gather(const void* ring, const int64_t* rpos, const int64_t* nval, int slots, int C,
                                      int H, const int64_t* rows, int B, void* out, void* stream) {
  if (!ring || !rpos || !nval || !rows || !out || slots <= 0 || C <= 0 || H <= 0 || B < 0) return CFB_ERR_INVALID_ARG;
  if (C > kRingMaxRows) return CFB_ERR_UNSUPPORTED;
  if ((H & 7) == 0 && ((reinterpret_cast<uintptr_t>(ring) | reinterpret_cast<uintptr_t>(out)) & 15))
    return CFB_ERR_INVALID_ARG;
  if (B == 0) return CFB_OK;
  ring_gather_kernel<<<B, kRingThreads, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const __half*>(ring), rpos, nval, C, H, rows, static_cast<__half*>(out));
  return cfb_launch_status("ring_gather_kernel");
}
