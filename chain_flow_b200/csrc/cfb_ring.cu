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

__device__ __forceinline__ void copy_row(__half* dst, const __half* src, int H) {
  if ((H & 7) == 0) {
    for (int c = threadIdx.x * 8; c < H; c += blockDim.x * 8)
      *reinterpret_cast<uint4*>(dst + c) = *reinterpret_cast<const uint4*>(src + c);
  } else {
    for (int c = threadIdx.x; c < H; c += blockDim.x) dst[c] = src[c];
  }
}

// Row j < kmax of request b is sh[start_b + off_j] (clamped into sh): off_j = j on a chain
// step; 0 for the committed token, then 1 + path[rows_b][j - 1] for the accepted tree nodes.
// Valid rows (j < cnt_b, wmask_b) go to position (rpos + j) mod C, the others to the trash row
// (with sh row 0, as the reference's masked index does); then rpos advances by cnt_b and nval
// saturates at C (only for wmask_b).
__global__ void __launch_bounds__(128) ring_write_kernel(__half* ring, int64_t* rpos, int64_t* nval, int C, int H,
                                                         const __half* sh, long long nsh, const int64_t* rows,
                                                         const int64_t* starts, const int64_t* cnt,
                                                         const uint8_t* wmask, const int64_t* path,
                                                         long long path_ld, int kmax) {
  const int b = blockIdx.x;
  const long long r = rows[b];
  const long long head = rpos[r];
  const long long n = cnt[b];
  const bool on = wmask[b] != 0;
  for (int j = 0; j < kmax; ++j) {
    const long long off = path ? (j == 0 ? 0 : 1 + path[r * path_ld + j - 1]) : j;
    const bool valid = j < n && on;
    long long src = 0;
    if (valid) src = min(max(starts[b] + off, 0ll), nsh - 1);
    const long long dst = valid ? (head + j) % C : C;
    copy_row(ring + (r * (C + 1) + dst) * H, sh + src * H, H);
  }
  __syncthreads();                                       // every thread has read rpos / nval
  if (threadIdx.x == 0) {
    const long long add = on ? n : 0;
    rpos[r] = (head + add) % C;
    nval[r] = min(nval[r] + add, (long long)C);
  }
}

// out[b, j] = ring[rows_b, (rpos - m + t) mod C], t = min(max(j - (C - m), 0), max(m - 1, 0)),
// m = nval[rows_b]: the slot's rows oldest first, front-padded by repeating the oldest one.
__global__ void __launch_bounds__(128) ring_gather_kernel(const __half* ring, const int64_t* rpos,
                                                          const int64_t* nval, int C, int H, const int64_t* rows,
                                                          __half* out) {
  const int b = blockIdx.x;
  const long long r = rows[b];
  const long long m = nval[r], head = rpos[r];
  for (int j = 0; j < C; ++j) {
    const long long t = min(max((long long)j - (C - m), 0ll), max(m - 1, 0ll));
    const long long phys = (((head - m + t) % C) + C) % C;
    copy_row(out + ((long long)b * C + j) * H, ring + (r * (C + 1) + phys) * H, H);
  }
}

}  // namespace

extern "C" cfb_status cfb_ring_write(void* ring, int64_t* rpos, int64_t* nval, int slots, int C, int H,
                                     const void* sh, int64_t nsh, const int64_t* rows, const int64_t* starts,
                                     const int64_t* cnt, const uint8_t* wmask, const int64_t* path,
                                     int64_t path_ld, int B, int kmax, void* stream) {
  if (!ring || !rpos || !nval || !sh || !rows || !starts || !cnt || !wmask || slots <= 0 || C <= 0 || H <= 0 ||
      nsh <= 0 || B < 0 || kmax <= 0 || (path && path_ld < kmax - 1))
    return CFB_ERR_INVALID_ARG;
  if ((H & 7) == 0 && ((reinterpret_cast<uintptr_t>(ring) | reinterpret_cast<uintptr_t>(sh)) & 15))
    return CFB_ERR_INVALID_ARG;
  if (B == 0) return CFB_OK;
  ring_write_kernel<<<B, 128, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<__half*>(ring), rpos, nval, C, H, static_cast<const __half*>(sh), nsh, rows, starts, cnt, wmask,
      path, path_ld, kmax);
  return cfb_launch_status("ring_write_kernel");
}

extern "C" cfb_status cfb_ring_gather(const void* ring, const int64_t* rpos, const int64_t* nval, int slots, int C,
                                      int H, const int64_t* rows, int B, void* out, void* stream) {
  if (!ring || !rpos || !nval || !rows || !out || slots <= 0 || C <= 0 || H <= 0 || B < 0) return CFB_ERR_INVALID_ARG;
  if ((H & 7) == 0 && ((reinterpret_cast<uintptr_t>(ring) | reinterpret_cast<uintptr_t>(out)) & 15))
    return CFB_ERR_INVALID_ARG;
  if (B == 0) return CFB_OK;
  ring_gather_kernel<<<B, 128, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const __half*>(ring), rpos, nval, C, H, rows, static_cast<__half*>(out));
  return cfb_launch_status("ring_gather_kernel");
}
