// cfb_pack.cu -- one-time weight preparation kernels of libcfb.so (run at drafter load).
//
// Packing replaces the reference's per-expert fp16 weight packing (reference
// src/chain_flow/cuda_block.py:266-311) with the streaming layout the engine reads: tiles of 64
// output rows, each [K/64][64 rows][128 B]; a 128-byte row holds 64 consecutive k of one output
// row with its 16-byte chunks XOR-swizzled by (row & 7). Each 8 KiB [64 x 64] block is the
// shared-memory image of a K-major, 128-byte-swizzled tcgen05 operand, and the two blocks of a
// 128-k streamed unit are contiguous, so the engine moves a unit with one bulk copy and the
// tensor cores read it in place. LayerNorm gamma is folded into the weight columns here;
// cfb_fold_bias folds beta into the bias and sums the folded columns.
#include <cuda_runtime.h>
#include <cuda_fp16.h>
#include <cstdint>
#include <cstdio>

#include "../../include/cfb.h"
#include "cfb_common.cuh"

namespace {

__global__ void pack_kernel(const __half* __restrict__ w, int64_t ldw, const int64_t* __restrict__ rows,
                            int nout, int k, const float* __restrict__ gamma, uint4* __restrict__ dst,
                            int ktotal, int kofs) {
  const int Mt = (nout + 63) / 64, nch = k / 8;
  const size_t tile_bytes = (size_t)64 * ((ktotal + 63) / 64 * 64) * 2;
  const long long n = (long long)Mt * 64 * nch;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n;
       i += (long long)gridDim.x * blockDim.x) {
    const int ch = (int)(i % nch), row = (int)(i / nch);
    __half h[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      const int col = ch * 8 + e;
      float v = 0.f;
      if (row < nout) {
        const int64_t src = rows ? rows[row] : row;
        v = __half2float(w[src * ldw + col]);
        if (gamma) v *= gamma[col];
      }
      h[e] = __float2half_rn(v);
    }
    const int k0 = kofs + ch * 8, m = row & 63, c = (k0 & 63) >> 3;
    const size_t byte = (size_t)(row >> 6) * tile_bytes + (size_t)(k0 >> 6) * 8192 + (size_t)m * 128 +
                        (size_t)((c ^ (m & 7)) << 4);
    dst[byte / 16] = *reinterpret_cast<const uint4*>(h);
  }
}

__global__ void fold_bias_kernel(const __half* __restrict__ w, int64_t ldw, int nout, int k,
                                 const float* __restrict__ gamma, const float* __restrict__ beta,
                                 const float* __restrict__ bias, float* __restrict__ out,
                                 float* __restrict__ colsum) {
  const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
  if (warp >= nout) return;
  float s = 0.f, c = 0.f;
  for (int j = lane; j < k; j += 32) {
    const float wv = __half2float(w[(int64_t)warp * ldw + j]);
    if (beta) s += wv * beta[j];
    c += __half2float(__float2half_rn(gamma ? wv * gamma[j] : wv));
  }
  for (int off = 16; off > 0; off >>= 1) {
    s += __shfl_xor_sync(0xffffffffu, s, off);
    c += __shfl_xor_sync(0xffffffffu, c, off);
  }
  if (lane == 0) {
    out[warp] = s + (bias ? bias[warp] : 0.f);
    if (colsum) colsum[warp] = c;
  }
}

__global__ void time_embed_kernel(const float* __restrict__ w1, const float* __restrict__ b1,
                                  const __half* __restrict__ w2, const float* __restrict__ b2, int D,
                                  int steps, float* __restrict__ out) {
  extern __shared__ float hsm[];
  const int s = blockIdx.y;
  const float tau = (float)s / (float)steps;
  for (int j = threadIdx.x; j < D; j += blockDim.x) {
    const float a = w1[j] * tau + b1[j];
    hsm[j] = a / (1.f + expf(-a));          // SiLU
  }
  __syncthreads();
  const int lane = threadIdx.x & 31, nw = blockDim.x >> 5;
  for (int i = blockIdx.x * nw + (threadIdx.x >> 5); i < D; i += gridDim.x * nw) {
    float acc = 0.f;
    for (int j = lane; j < D; j += 32) acc += __half2float(w2[(int64_t)i * D + j]) * hsm[j];
    for (int off = 16; off > 0; off >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, off);
    if (lane == 0) out[(int64_t)s * D + i] = acc + b2[i];
  }
}

}  // namespace

extern "C" {

size_t cfb_packed_bytes(int nout, int k) {
  if (nout <= 0 || k <= 0 || k % 16) return 0;
  return (size_t)((nout + 63) / 64) * 64u * (size_t)((k + 63) / 64 * 64) * 2u;
}

cfb_status cfb_pack_linear(const void* w, int64_t ldw, const int64_t* rows, int nout, int k,
                           const float* gamma, void* dst, int ktotal, int kofs, void* stream) {
  if (!w || !dst || nout <= 0 || k <= 0 || k % 16 || ktotal % 16 || kofs % 16 || kofs + k > ktotal ||
      ldw < k)
    return CFB_ERR_INVALID_ARG;
  if (reinterpret_cast<uintptr_t>(dst) % 16) return CFB_ERR_INVALID_ARG;
  const long long n = (long long)((nout + 63) / 64) * 64 * (k / 8);
  const int threads = 256;
  const int blocks = (int)((n + threads - 1) / threads < 65535 ? (n + threads - 1) / threads : 65535);
  pack_kernel<<<blocks, threads, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const __half*>(w), ldw, rows, nout, k, gamma, static_cast<uint4*>(dst), ktotal, kofs);
  return cfb_launch_status("pack_kernel");
}

cfb_status cfb_fold_bias(const void* w, int64_t ldw, int nout, int k, const float* gamma,
                         const float* beta, const float* bias, float* bias_out, float* colsum_out,
                         void* stream) {
  if (!w || !bias_out || nout <= 0 || k <= 0 || ldw < k) return CFB_ERR_INVALID_ARG;
  const int threads = 256, blocks = (int)(((long long)nout * 32 + threads - 1) / threads);
  fold_bias_kernel<<<blocks, threads, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const __half*>(w), ldw, nout, k, gamma, beta, bias, bias_out, colsum_out);
  return cfb_launch_status("fold_bias_kernel");
}

cfb_status cfb_time_embed(const float* w1, const float* b1, const void* w2_f16, const float* b2,
                          int D, int steps, float* out, void* stream) {
  if (!w1 || !b1 || !w2_f16 || !b2 || !out || D <= 0 || steps <= 0) return CFB_ERR_INVALID_ARG;
  if ((size_t)D * sizeof(float) > 48 * 1024) return CFB_ERR_UNSUPPORTED;
  time_embed_kernel<<<dim3(32, steps), 256, D * sizeof(float), static_cast<cudaStream_t>(stream)>>>(
      w1, b1, static_cast<const __half*>(w2_f16), b2, D, steps, out);
  return cfb_launch_status("time_embed_kernel");
}

}  // extern "C"
