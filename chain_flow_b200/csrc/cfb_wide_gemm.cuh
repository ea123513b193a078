// cfb_wide_gemm.cuh -- the batched ("wide") drafting path's GEMM: C = A · Wᵀ on the 5th-generation
// tensor cores of sm_100a.
//
// A is an fp16 activation matrix [M, K], row-major (K-major). W, an fp16 weight matrix [N, K], is
// stored tiled (cfb_wide_pack): [N/256][K/64] blocks of 256 rows x 64 columns, 32 KiB each,
// contiguous, every block already in the 128-byte-swizzled shared-memory image the tensor cores
// read, so a CTA streams its weights as consecutive 32 KiB bulk copies, while the activations,
// re-read from L2 by every CTA of a row of tiles, come in through 2-D TMA.
// One CTA computes a 256 × 256 output tile (two 128-row M tiles of activations × 256 weight
// rows; one M tile where M ends) over one k range (split-K): each weight block it streams feeds
// both M tiles, so the weights are read once per 256 activation rows. 192 threads in three roles:
//   warp 0, one lane   producer: per stage one 2-D tiled TMA copy of each 128 × 64 A tile (128-byte
//                      swizzle) and one 32 KiB bulk copy of the W block into the stage ring;
//   warp 1             allocates 512 TMEM columns (two fp32 accumulators); one lane issues
//                      tcgen05.mma (M = 128, N = 256, K = 16, four per stage and M tile) and
//                      returns each stage to the producer with tcgen05.commit;
//   warps 2..5         epilogue: each thread owns one accumulator row (its TMEM lane), reads it
//                      16 columns at a time with tcgen05.ld and applies the fused epilogue.
// Every wait is bounded: the ring waits by the launch's budget (default kWaitBudgetNs), the waits
// that let the CTA wind down by kWaitBudgetNs. A ring wait that expires records an error and the
// CTA winds down: the accumulator wait still lets every issued MMA finish, the producer waits for
// its copies in flight, and TMEM is always freed.
#pragma once
#include <cuda.h>
#include "cfb_common.cuh"

namespace cfb {
namespace wide {

constexpr int BM = 128, BN = 256, BK = 64;
constexpr int kGemmThreads = 192;
constexpr uint32_t kTileBytes = BM * BK * 2;             // 16 KiB A tile (128 rows)
constexpr uint32_t kWTileBytes = BN * BK * 2;            // 32 KiB W block
// a CTA covers one or two 128-row M tiles: stages of 2 x 16 + 32 = 64 KiB (3 deep) or
// 16 + 32 = 48 KiB (4 deep); two fp32 accumulators of 256 columns fill the 512 TMEM columns
constexpr int kMaxStages = 4;
constexpr uint32_t kRingBytes = 192 * 1024;
constexpr size_t kGemmSmem = kRingBytes + 1024 /* 1 KiB alignment slack */ + 256;
constexpr int kTopMaxW = 8;                              // head epilogue: longest top list

enum EpiKind : int {
  EPI_F32 = 0,      // out32[r, c] = acc + bias                      (tests, partials)
  EPI_F16 = 1,      // out16[r, c] = fp16(acc + bias)
  EPI_GELU16 = 2,   // out16[r, c] = fp16(gelu(acc + bias))
  EPI_PART = 3,     // part[split][r, c] = acc                       (split-K residual GEMMs)
  EPI_EULER = 4,    // z[b, start + r % chunk, c] += dt * (acc + bias), b = r / chunk
  EPI_PATH = 5,     // out32[r, c] = acc + sum_{j < nlive, lastp[r][j] >= 0} pbias[j, c]
  EPI_HEADIN = 6,   // out16[r, c] = fp16(acc + bias + pred[r / beams, step, c])
  EPI_HEAD = 7      // per (row, tile): online (max, sum exp) and top-`topb` (value, id)
};

struct GemmProb {
  CUtensorMap ta;                 // A [M, K]: box 64 × 128
  const __half* wt;               // W, tiled: block (n tile, k block) at (nt * kbt + kb) * BN * BK
  int kbt;                        // k blocks of the packed W (its full K / 64)
  int M, N, kblocks;              // kblocks = K / 64 actually multiplied
  int m_tiles, n_tiles, splits, kb_per_split;
  int pair;                       // 1: a CTA covers M tiles 2 mp and 2 mp + 1; 0: M tile mp only
  int m_pairs;                    // CTAs along M
  int cta0;                       // first CTA of this problem in the grouped launch
  int epi;
  const float* bias;              // [N] or null
  void* out;                      // epilogue target (see EpiKind)
  long long ldo;                  // row stride of `out` in elements
  long long split_stride;         // EPI_PART: elements between two splits' partials
  // EPI_EULER
  float dt; int chunk, zrows, zstart;
  // EPI_PATH
  const int64_t* lastp; int order, nlive; const float* pbias;
  // EPI_HEADIN
  const float* pred; int beams, pred_rows, step;
  // EPI_HEAD
  int topb, rowoff;
  // split-K of a non-partial epilogue: each split stores its fp32 tile to fix_ws
  // [tile][split][BM][BN]; the split that arrives last at fix_cnt[tile] adds them in split order,
  // applies the epilogue and resets the counter (nobody waits)
  float* fix_ws; int* fix_cnt;
};

constexpr int kMaxProbs = 8;
struct GemmLaunch {
  GemmProb p[kMaxProbs];
  int nprob;
  int* err;                       // sticky device error word
  unsigned long long wait_ns;     // budget of the ring waits (cfb_run.wait_budget_ns; default 1 s)
};
static_assert(sizeof(GemmLaunch) <= 4000, "kernel parameter space");

// ---- PTX wrappers: TMA, tcgen05 ---------------------------------------------------------------
CFB_DEV void tma_load_2d(void* smem_dst, const CUtensorMap* map, int x, int y, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];"
      :: "r"(smem_u32(smem_dst)), "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_u32(bar))
      : "memory");
}
CFB_DEV void prefetch_tmap(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" :: "l"(reinterpret_cast<uint64_t>(map)) : "memory");
}
// Instruction descriptor: fp32 accumulator, fp16 A and B, both K-major, M = 128, N = 256.
constexpr uint32_t kIdesc = (1u << 4) | ((uint32_t)(BN >> 3) << 17) | ((uint32_t)(BM >> 4) << 24);

CFB_DEV bool better_w(float v, int i, float w, int j) { return v > w || (v == w && i < j); }

}  // namespace wide
}  // namespace cfb
