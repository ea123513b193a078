// cfb_engine.cu -- the persistent drafting engine of libcfb.so (sm_100a).
//
// One cooperative launch runs a whole draft: the flow integrator (both chunk experts, every
// HiddenKVFlowBlock, every Euler step, cross-K/V hoisted once per draft), then per draft depth
// the path residual, the markov-bias gather, the shortlist head with online log-sum-exp + top-k
// (no logits reach HBM) and the beam step. The host side (cfb_plan_build, C++ below) lowers a
// (drafter, run) pair into a table of phases; the kernel walks the table with a bounded grid
// barrier between phases.
//
// Each CTA is warp-specialised:
//   * weight producer (1 thread): streams the CTA's packed weight units of every GEMM phase
//     (64 output features x 128 k, 16 KiB) into a shared-memory ring with cp.async.bulk (the
//     TMA copy engine, no multicast), running ahead across phase boundaries since weights never
//     depend on activations;
//   * activation producer (1 warp): once the grid barrier in front of a phase has passed,
//     copies each unit's activation rows into the same ring slot with 16-byte cp.async;
//   * 8 MMA warps: multiply each unit with tensor-core MMAs and, at the end of a 64-feature
//     tile, hand their fp32 partials to a shared-memory slot and move on;
//   * 4 epilogue warps: reduce the 8 partials in a fixed order, complete tiles split across
//     CTAs (stream-K: whichever CTA arrives last sums the partials in k order -- deterministic,
//     no float atomics), apply the fused epilogue (bias, LayerNorm correction, GELU, residual,
//     Euler step, row statistics, attention of completed heads, head log-sum-exp + top-k) and
//     take the beam step.
//
// A LayerNorm in front of a linear is folded at pack time (W <- W diag(gamma), b <- b + W beta);
// the engine feeds the fp16 activation straight into the MMA and applies
//     y = (acc - mean * colsum(W)) * rstd + b
// in the epilogue, with the row statistics combined from per-64-column parts that the producing
// epilogue wrote (Chan's parallel mean/M2 merge, fixed order).
//
// Reference behaviour restated (paths relative to the reference checkout):
//   HiddenKVFlowBlock            src/chain_flow/drafters/chunked_flow.py:168-202
//   HiddenKVFlowExpert pre/post  src/chain_flow/drafters/chunked_flow.py:333-414
//   Euler integrate / chunks     src/chain_flow/drafters/tree_flow.py:163-235
//   path residual                src/chain_flow/drafters/tree_flow.py:434-450
//   head / bias / map / beams    src/chain_flow/vllm_plugin/flow_proposer.py:1021-1028, 1188-1332
#include <cuda_runtime.h>
#include <cuda_fp16.h>
#include <cstdint>
#include <cstring>
#include <cstdlib>
#include <cmath>
#include <cstdio>
#include <vector>
#include <algorithm>
#include <mutex>
#include <type_traits>

#include "cfb_common.cuh"
#include "../../include/cfb.h"

namespace cfb {

// ---- thread layout: [0,8) worker warps (in GEMM phases warp 0 issues the tensor-core MMAs; all
// 8 take part in the other phases' work), 8 weight producer, 9 activation producer, [10,14)
// epilogue.
constexpr int kMmaWarps = 8;
constexpr int kMmaIssueWarp = 0;
constexpr int kMma = kMmaWarps * 32;                // 256
constexpr int kWProdWarp = 8, kXProdWarp = 9, kEpiWarp0 = 10;
constexpr int kEpiWarps = 4;
constexpr int kEpi = kEpiWarps * 32;                // 128
constexpr int kThreads = (kMmaWarps + 2 + kEpiWarps) * 32;   // 448
constexpr int kWorkers = kMma + kEpi;               // threads that take part in phase-level work
constexpr int kBarWorkers = 1, kBarEpi = 2;         // named barriers (0 is __syncthreads)
// GEMM phases of the wide-row builds (engine_kernel<4|8>): worker warps 1..7, idle there, join
// the epilogue warps for everything but the accumulator readout
constexpr int kBarWide = 11;                        // (3..10 are the beam merge's row groups)
constexpr int kEpiWide = kEpi + (kMmaWarps - 1) * 32;   // 352

constexpr int kTileRows = 64;                       // output features per tile (the MMA's M)
constexpr int kUnitK = 8;                           // 16-wide k blocks per streamed unit
constexpr int kBlockBytes = 512;                    // 64 features x 16 k x fp16 of packed weights
constexpr int kUnitBytes = 4 * kUnitK * kBlockBytes;    // 16 KiB: two 8 KiB [64 x 64] halves
constexpr int kHalfBytes = kUnitBytes / 2;
constexpr int kAccCols = 64;                        // TMEM columns of one accumulator (N <= 64 rows)
constexpr int kMaxStages = 12;
constexpr int kSmemBudget = 232448 - 1024 - 2048;   // dynamic + static shared memory per CTA
constexpr int kRowsMax = 64;                        // activation rows per job
constexpr int kTopMax = 8;                          // top-k per beam row
constexpr int kMaxExperts = 4;
constexpr int kStatCols = 64;                       // columns per row-statistics part
constexpr int kHeadPartFloats = 2 + 2 * kTopMax;
static_assert(kRowsMax == CFB_XROWS && kHeadPartFloats == CFB_XFLOATS, "xloc layout of cfb.h");
constexpr int kMaxSeg = 16;
// Descriptor cache: the activation producer copies each phase's record and (up to kJobCache)
// jobs into one of kDescBufs shared-memory slots a phase ahead, so that the roles do not wait on
// the job table in global memory after a grid barrier (whose acquire leaves the L1 cold).
constexpr int kJobCache = 4, kDescBufs = 3, kPhaseSlot = 64;                         // launch segments of a plan (sharded heads)

enum XKind : int { XK_F16 = 0 };

// fp16 activations the engine produces for its own GEMMs are stored tiled: each 64-column slice
// of all R rows is contiguous, one 128-byte row per activation row, its 16-byte chunks XOR-
// swizzled by (row & 7). A slice copied to a 1024-byte-aligned shared-memory address is then the
// K-major, 128-byte-swizzled B operand of tcgen05.mma as it stands; a streamed unit (128 k) takes
// two bulk copies. Element (r, k) of an R-row buffer:
CFB_DEV size_t tidx(int R, int r, int k) {
  return ((size_t)(k >> 6) * R + r) * 64 + (size_t)((((k & 63) >> 3) ^ (r & 7)) << 3) + (k & 7);
}
enum LnKind : int { LN_NONE = 0, LN_PARTS = 1, LN_DIRECT = 2 };
enum EKind : int { EK_STORE = 0, EK_GELU16 = 1, EK_RESID = 2, EK_EULER = 3, EK_PATHH = 4,
                   EK_HEADIN = 5, EK_HEAD = 6, EK_STORE16 = 7 };
// the plan mode of a VAE side (cfb_vae_plan_build): not a cfb_mode the caller can ask for
constexpr int kModeVae = 16;
enum PKind : int { PK_PREP = 0, PK_GEMM = 1, PK_ATTN = 2, PK_BEAM = 3, PK_RMERGE = 4, PK_GATHER = 5,
                   PK_TPXA = 6, PK_TPSEL = 7, PK_TPGATH = 8, PK_TPKEY = 9, PK_TPRAD = 10,
                   PK_TPCNT = 11 };   // 6-11: the two-pass head
enum Post : int { PO_NONE = 0, PO_BEAM_CHAIN = 1, PO_BEAM_TREE = 2, PO_PUBLISH = 3 };

// Attention of one (expert, block): q rows [B*Sq] and k/v rows [B*Kn] (fp32, written by the
// projection phase before it), output fp16 tiled with outR rows. One task = (request, head).
struct alignas(16) AttnTask {
  const float* q; int ldq, qoff;
  const float* k; int ldk, koff;
  const float* v; int ldv, voff;
  __half* out;
  int rows_per_req, keys_per_req, B, hd, heads, causal;
  float scale;
  int outR;               // tiled rows of `out`
};

struct ExpertRT {
  float* x32[2]; __half* x16[2]; float2* xstat[2];   // residual stream, by Euler step parity
  int S; int start;
  const float* pos; const float* temb;
};

struct alignas(16) Job {
  const uint4* w;
  int Mt, Kt, Kstride, nkc, rows, nout;
  int unit_base, tile_base;
  // activation source (fp16 rows, or a gather of embedding rows by path token)
  int xkind;
  const __half* x; int ldx;                // tiled source with xR rows
  int xR, xcopy;                           // tiled rows of the source; rows copied per unit
  int gin, gstride, goff;                  // source row = (r / gin) * gstride + goff + r % gin
  int ln; const float2* stats; int nparts; const float* colsum;
  int order; int D;                        // EK_PATHH: path order, hidden size
  // epilogue
  int ekind;
  const float* bias;
  float* out32; __half* out16; int ldo; int oR;   // out32 row stride; out16 tiled rows
  float2* ostats; int onparts;
  int e_idx, step, last_step, wrows, nlive, R, topb;
  int rowoff;                              // EK_HEAD: shortlist row of the head's first row
  // EK_HEAD of the two-pass head: pass A stores the raw scores [rows, R] (logits); pass B maps
  // column c to shortlist row cand[c] and scores row r only against the columns of its own
  // request (c / cmask == r / wrows)
  float* logits; const int* cand; int cmask;
  float dt;
  const float* p0;                         // EK_PATHH: offset biases [order][D]
};

// a CFB_BUF_PHASES record (layout documented in cfb.h): int fields only
struct Phase {
  int kind;
  int job0, njobs, nunits, ntiles;   // PK_ATTN: job0 / njobs index attention tasks, ntiles = tasks
  int whole;                // 1: each CTA gets whole tiles (no cross-CTA fixups); 0: stream-K
  int post;
  int step, rows, fr, keep, topb, base, base_prev, last;
};
static_assert(sizeof(Phase) == 15 * sizeof(int), "CFB_BUF_PHASES record");
// Phase.last of a GEMM phase (unused by GEMM phases otherwise): its weights are written by an
// earlier phase of the same launch, so the weight producer may stream them only once the workers
// have entered the phase
constexpr int kWeightsWritten = 2;
static_assert(sizeof(Phase) <= kPhaseSlot, "descriptor cache slot");
static_assert(sizeof(Job) % 16 == 0 && kJobCache * sizeof(Job) / 16 <= 64, "descriptor cache copy");
static_assert(sizeof(AttnTask) % 16 == 0, "descriptor cache copy");
// attention tasks a descriptor cache slot holds (in the room of its jobs)
constexpr int kAttnCache = (int)(kJobCache * sizeof(Job) / sizeof(AttnTask));

// The cost of a cross-CTA split-tile fixup (publish, owner's bounded wait, sum), in streamed
// units, for the whole-tiles-or-split choice of each GEMM phase.
#ifndef CFB_FIXUP_UNITS
#define CFB_FIXUP_UNITS 12
#endif
// The same for jobs of more than 16 rows: a contributor's published partial and the owner's sum
// grow with the rows, and the fixup then measured dearer.
#ifndef CFB_FIXUP_UNITS_WIDE
#define CFB_FIXUP_UNITS_WIDE 24
#endif

// Dynamic shared memory, laid out per plan by the host from a 1024-byte-aligned base: the ring of
// streamed units (each stage = 16 KiB of packed weights + the unit's activation rows as two
// [xhalf / 128 rows][128 B] halves), mbarriers, a staging tile for accumulators whose rows are
// gathered, the epilogue's scratch (attention / merge ids), one reduced tile, row statistics.
struct SmemLayout {
  int nstages, stage_bytes, rows_pad, nbuf, xhalf;
  int off_bar, off_slots, off_scratch, off_red, off_rowstat, off_tile, off_misc, off_desc, total;
};

struct Plan {
  SmemLayout sm;
  int G, nphases, mode, B, D, DL, n_experts, chunk, C, steps, order, rank, vocab, R;
  int width, depth, keep, topb, Wmax, N;
  const Phase* phases;
  const Job* jobs;
  const AttnTask* attn;
  ExpertRT ex[kMaxExperts];
  unsigned* bar; unsigned* exitcnt; int* err;
  unsigned* tilecnt; int ntilecnt;
  float* gpart;             // [G][kTileRows*kRowsMax]: each CTA's one published split-tile partial
  float* hpart;             // [G][kRowsMax][kHeadPartFloats]
  const __half* ctx; const __half* z0; float* pred; float2* ctxstat; __half* ctx16;
  int init_mode;            // CFB_INIT_GIVEN / REPEAT_LAST / DELTA
  const int64_t* known0; int64_t* lastp; float* cum; int64_t* toks; int* bps; int64_t* tokens;
  const int64_t* shortlist; const __half* markov_w1; __half* xhead; int ldxhead;
  const __half* emb; __half* pg;            // embeddings; tiled path-gather rows of the path GEMM
  int nranks; const float* xall; float* xloc;   // row-sharded head: gathered / local merged lists
  int nseg; int seg[kMaxSeg + 1];           // launch segments: phases [seg[i], seg[i + 1])
  int maxnt;                                // engine_kernel<maxnt> runs this plan
  void* buf[16]; size_t buf_bytes[16];     // intermediate buffers exposed by cfb_plan_buffer
  unsigned long long* prof;                // [nphases][G][4] or NULL
  unsigned long long wait_ns;              // the grid barrier's wait budget (cfb_run.wait_budget_ns)
  // a VAE side (mode kModeVae): input rows [B * vS, vDin] (fp32 when vin32, else fp16), unit-
  // tiled into vin16 by prep; the residual stream vx32 [B * vS, D] starts at pos[row % vS]
  const void* vin; int vin32, vS, vDin;
  __half* vin16; float* vx32; const float* vpos;
  // the two-pass head (tp_m > 0): tp_n marginal rows per request (depths 1..tp_n), their fp16
  // head input txa, pass A's scores tlog [B * tp_n, R], the candidates' keys tkeys [B, R], the
  // candidate set tcd [B, tp_m] (shortlist rows, ascending) and its packed head rows tchead
  int tp_m, tp_n, tp_rs;    // tp_rs: the key rows' stride (R rounded up to 4)
  unsigned* thist;          // [4][B][256] radix histograms of the keys, one byte per pass
  int* tcnt;                // [B][G][2] per-CTA counts of keys above / at the threshold
  const uint4* tp_head;     // the packed full shortlist head the candidates are read from
  __half* txa; float* tlog; unsigned* tkeys; int* tcd; uint4* tchead;
};

struct Smem {
  uint8_t* ring; int nstages, stage_bytes, rp, nbuf, xhalf;
  uint64_t* full; uint64_t* empty;         // per ring stage
  uint64_t* accf; uint64_t* acce;          // per TMEM accumulator buffer
  uint64_t* fin;                           // the MMA warp's last commit (before TMEM is freed)
  uint32_t tmem;                           // TMEM base: nbuf accumulators of kAccCols columns
  float* slots;                            // [kTileRows][kAccCols + 1]: accumulator staging
  float* scratch;                          // attention / merge ids (epilogue only)
  float* red;                              // [kTileRows][rp]
  float2* rowstat;
  float* tbias; float* tcsum;              // [kTileRows] bias / LayerNorm column sums of the tile
  int* flag;
  volatile int* phase_ready;               // the phase the workers have entered
  volatile int* desc_ready;                // the last phase whose descriptors are cached
  uint8_t* desc;                           // kDescBufs x (phase record slot + kJobCache jobs)
  __device__ const Phase& dphase(int p) const {
    return *reinterpret_cast<const Phase*>(desc + (size_t)(p % kDescBufs) * (kPhaseSlot + kJobCache * sizeof(Job)));
  }
  __device__ const Job* djobs(int p) const {
    return reinterpret_cast<const Job*>(desc + (size_t)(p % kDescBufs) * (kPhaseSlot + kJobCache * sizeof(Job)) + kPhaseSlot);
  }
  __device__ uint8_t* stage(int s) const { return ring + (size_t)s * stage_bytes; }
};

// A cooperating thread group: index in group, size, named barrier.
struct Grp { int t, n, bar; };
CFB_DEV void gsync(const Grp& g) { asm volatile("bar.sync %0, %1;" :: "r"(g.bar), "r"(g.n) : "memory"); }

struct HeadState { float m, s; float tv[kTopMax]; int ti[kTopMax]; };

// Profiling (plans built with CFB_RUN_PROFILE): ns spent waiting, per role, reset every phase,
// and the times of a few events (the layout of a CFB_BUF_PROF record is documented in cfb.h).
constexpr int kProfSlots = 20;
// Two clock types: plans built with CFB_RUN_PROFILE run the engine instantiation with ProfClock;
// every other plan gets NoClock, whose fields are never touched (every use sits under `if
// (wc.on)`), so unprofiled kernels spend no registers on profiling.
struct ProfClock {
  unsigned long long full = 0, slot = 0;
  unsigned long long first = 0, last = 0;   // when the phase's first / last unit was ready
  unsigned long long part = 0, atom = 0, fix = 0, tdone = 0;   // epilogue: last tile's events
  unsigned long long rstat = 0;                                // epilogue: row statistics loaded
  bool on = false;
  CFB_DEV unsigned long long now() const { return on ? globaltimer() : 0ull; }
};
struct NoClock {
  unsigned long long full, slot, first, last, part, atom, fix, tdone, rstat;
  static constexpr bool on = false;
  CFB_DEV unsigned long long now() const { return 0ull; }
};

// ------------------------------------------------------------------------------------------
// The grid barrier counter's top bit: set with the error word, so that every CTA waiting at (or
// arriving at) a grid barrier sees the failure in the value it polls anyway.
constexpr unsigned kBarErrBit = 0x80000000u;
CFB_DEV void set_err(const Plan& P, int code) {
  atomicCAS(P.err, 0, code);
  atomicOr(P.bar, kBarErrBit);
}

// 32-bit arithmetic: plans are only built when U * (G + 1) fits in 32 bits
CFB_DEV long long cta_start(long long U, int G, int c) {
  return (long long)((unsigned)c * (unsigned)U / (unsigned)G);
}
CFB_DEV int cta_of(long long u, long long U, int G) {       // the CTA whose range holds unit u
  return (int)((((unsigned)u + 1u) * (unsigned)G + (unsigned)U - 1u) / (unsigned)U) - 1;
}
// the next CTA after c whose (non-empty) range holds units; CTAs with empty ranges are skipped
CFB_DEV int next_contributor(int c, long long U, int G) {
  return cta_of(cta_start(U, G, c + 1), U, G);
}

// grid barrier over the worker threads of all CTAs; bounded; false once an error is set
// Thread-0 side of waiting for phase `next`'s cached descriptors (filled by the activation
// producer warp); false if the wait gave up or the plan failed.
CFB_DEV bool desc_wait1(const Plan& P, volatile int* desc_ready, int next) {
  if (*desc_ready >= next) { __threadfence_block(); return true; }
  const unsigned long long t0 = globaltimer();
  for (unsigned it = 1; *desc_ready < next; ++it) {
    if (it % kPollsPerCheck) continue;
    if (ld_volatile_int(P.err) != 0) return false;
    if (globaltimer() - t0 > kWaitBudgetNs) { set_err(P, DEV_TIMEOUT_SLOT); return false; }
  }
  __threadfence_block();
  return true;
}

// Grid barrier of the worker threads; then (next >= 0) phase `next`'s descriptors are cached.
CFB_DEV bool grid_sync(const Plan& P, unsigned& epoch, const Grp& W, volatile int* desc_ready, int next) {
  gsync(W);
  __shared__ int s_ok;
  if (W.t == 0) {
    ++epoch;
    // the CTA barrier above orders every thread's writes before this release (acq_rel) atomic
    const unsigned target = epoch * (unsigned)P.G;
    unsigned v = atom_add_acqrel(P.bar, 1u) + 1u;
    if (v < target) {
      const unsigned long long t0 = globaltimer();
      const unsigned every = polls_per_check(P.wait_ns);
      for (unsigned it = 1; (v = ld_acquire(P.bar)) < target; ++it) {
        if (it % every == 0 && wait_expired(t0, P.wait_ns)) {
          set_err(P, DEV_TIMEOUT_GRID);
          v = kBarErrBit;
          break;
        }
      }
    }
    bool good = (v & kBarErrBit) == 0u;
    if (good && next >= 0) good = desc_wait1(P, desc_ready, next);
    s_ok = good;
  }
  gsync(W);
  return s_ok != 0;
}

CFB_DEV int src_row(const Job& J, int r) { return (r / J.gin) * J.gstride + J.goff + r % J.gin; }

// ------------------------------------------------------------------------------------------
// LayerNorm statistics as (mean, M2 = sum of squared deviations) of equal-count groups, merged
// without divisions: for k groups of c values each, mean = avg(mean_g) and
// M2 = sum(M2_g) + c * sum((mean_g - mean)^2) (the pairwise form of Chan et al. with equal counts).

// (mean, M2) of 8 values, two-pass.
CFB_DEV void stats8(const float (&v)[8], float& mean, float& M2) {
  float sum = 0.f;
#pragma unroll
  for (int i = 0; i < 8; ++i) sum += v[i];
  mean = sum * 0.125f;
  float q = 0.f;
#pragma unroll
  for (int i = 0; i < 8; ++i) { const float d = v[i] - mean; q += d * d; }
  M2 = q;
}

// Fold group k (0-based; 8 values: mean mb, M2 qb) into the running statistics of groups 0..k-1.
CFB_DEV void stats8_add(float& m, float& M2, int k, float mb, float qb) {
  if (k == 0) { m = mb; M2 = qb; return; }
  const float r = k == 1 ? 0.5f : k == 2 ? (1.f / 3.f) : k == 3 ? 0.25f : 1.f / (float)(k + 1);
  const float d = mb - m;
  m += d * r;
  M2 += qb + d * d * (8.f * (float)k) * r;
}

// Merge equal-count statistics (cnt values each) held by `width` adjacent lanes (a power of two);
// every lane of the group ends with the same result (butterfly sums are order-independent here:
// each stage adds two identical partial values). Out of line, like job_rowstats: inlined, these
// measured 2-3 % slower weight streaming in the large phases (register allocation of the loop).
__device__ __noinline__ void eq_group(float& m, float& M2, float cnt, int width) {
  float s = m;
  for (int off = 1; off < width; off <<= 1) s += __shfl_xor_sync(0xffffffffu, s, off);
  const float mean = s * (1.f / (float)width);
  const float d = m - mean;
  float q = M2 + cnt * d * d;
  for (int off = 1; off < width; off <<= 1) q += __shfl_xor_sync(0xffffffffu, q, off);
  m = mean; M2 = q;
}

// Row LayerNorm statistics of the job's source rows -> S.rowstat[r] = (mean, rstd) (epilogue).
__device__ __noinline__ void job_rowstats(const Job& J, Smem& S, const Grp& E) {
  const int warp = E.t >> 5, lane = E.t & 31, nw = E.n >> 5;
  if (J.ln == LN_PARTS) {
    // the row's parts are kStatCols columns each: mean = avg(part means), then
    // M2 = sum(part M2 + kStatCols * (part mean - mean)^2); parts lane, lane + 32, ... per lane
    constexpr int kPL = 4;                                  // parts per lane (<= 128 parts)
    const int np = J.nparts;
    const float inv = 1.f / (float)np;
    for (int r = warp; r < J.rows; r += nw) {
      const int sr = src_row(J, r);
      float2 st[kPL];
      float ms = 0.f;
#pragma unroll
      for (int j = 0; j < kPL; ++j) {
        const int p = lane + 32 * j;
        st[j] = p < np ? __ldcg(J.stats + (size_t)sr * np + p) : make_float2(0.f, 0.f);
        ms += st[j].x;
      }
#pragma unroll
      for (int off = 16; off > 0; off >>= 1) ms += __shfl_xor_sync(0xffffffffu, ms, off);
      const float mean = ms * inv;
      float q = 0.f;
#pragma unroll
      for (int j = 0; j < kPL; ++j)
        if (lane + 32 * j < np) { const float d = st[j].x - mean; q += st[j].y + (float)kStatCols * d * d; }
#pragma unroll
      for (int off = 16; off > 0; off >>= 1) q += __shfl_xor_sync(0xffffffffu, q, off);
      if (lane == 0) S.rowstat[r] = make_float2(mean, rsqrtf(q * inv * (1.f / (float)kStatCols) + 1e-5f));
    }
  } else if (J.ln == LN_DIRECT) {
    for (int r = E.t; r < J.rows; r += E.n) S.rowstat[r] = __ldcg(J.stats + src_row(J, r));
  } else {
    for (int r = E.t; r < J.rows; r += E.n) S.rowstat[r] = make_float2(0.f, 1.f);
  }
  gsync(E);
}

// y = (acc - mean * colsum) * rstd + bias for feature f of the current tile, row r
CFB_DEV float epi_val(const Smem& S, int f, int r) {
  const float2 rs = S.rowstat[r];
  return (S.red[f * S.rp + r] - rs.x * S.tcsum[f]) * rs.y + S.tbias[f];
}

// Row/slice mapping of the epilogue threads for per-row work: `sl` threads per row (8, 4 or 2),
// each owning 64 / sl consecutive features of a 64-feature tile; whole warps take part.
struct RowMap { int r, q, sl, nf; };
CFB_DEV RowMap row_map(int rows, int et, int n) {
  const int rp = rows <= 16 ? 16 : rows <= 32 ? 32 : 64;
  const int per = n / rp;                                 // threads per row the group affords
  const int sl = per >= 8 ? 8 : per >= 4 ? 4 : 2;         // a power of two: 8 or more features each
  return {et / sl, et % sl, sl, kTileRows / sl};
}

// the head epilogue's map: a row gets kEpi / rows lanes (at least 2 features each), so small
// row counts keep every epilogue thread busy
CFB_DEV RowMap head_map(int rows, int et, int n) {
  const int rp = rows <= 4 ? 4 : rows <= 8 ? 8 : rows <= 16 ? 16 : rows <= 32 ? 32 : 64;
  const int per = n / rp;                                 // threads per row the group affords
  const int sl = per >= 32 ? 32 : per >= 16 ? 16 : per >= 8 ? 8 : per >= 4 ? 4 : 2;
  return {et / sl, et % sl, sl, kTileRows / sl};
}

// ------------------------------------------------------------------------------------------
// Attention of request b, head h (reference nn.MultiheadAttention inside HiddenKVFlowBlock,
// chunked_flow.py:185-197): softmax(q k^T * hd^-1/2 [+ causal mask]) v over the request's rows.
// Run by all worker warps of one CTA; q/k/v slices go to shared memory with one cp.async batch.
CFB_DEV void attn_task(const AttnTask& A, int b, int h, Smem& S, const Grp& W) {
  const int Sq = A.rows_per_req, Kn = A.keys_per_req, hd = A.hd;
  float* qs = S.scratch;
  float* ks = qs + Sq * hd;
  float* vs = ks + Kn * hd;
  float* sc = vs + Kn * hd;
  const int cpr = hd / 4;                       // 16-byte chunks per head row
  for (int e = W.t; e < (Sq + 2 * Kn) * cpr; e += W.n) {
    const int row = e / cpr, c = e - row * cpr;
    const float* src;
    float* dst;
    if (row < Sq) {
      src = A.q + (size_t)(b * Sq + row) * A.ldq + A.qoff + h * hd + c * 4;
      dst = qs + row * hd + c * 4;
    } else if (row < Sq + Kn) {
      const int j = row - Sq;
      src = A.k + (size_t)(b * Kn + j) * A.ldk + A.koff + h * hd + c * 4;
      dst = ks + j * hd + c * 4;
    } else {
      const int j = row - Sq - Kn;
      src = A.v + (size_t)(b * Kn + j) * A.ldv + A.voff + h * hd + c * 4;
      dst = vs + j * hd + c * 4;
    }
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" :: "r"(smem_u32(dst)), "l"(src) : "memory");
  }
  asm volatile("cp.async.commit_group;\n\tcp.async.wait_group 0;" ::: "memory");
  gsync(W);
  // scores: T adjacent lanes per (i, j) pair, each summing every T-th 4-column chunk
  const int pairs = Sq * Kn;
  int T = 32;
  while (T > 1 && pairs * T > W.n) T >>= 1;
  const int lane = W.t & 31, gl = lane & (T - 1);
  for (int p0 = 0; p0 < pairs * T; p0 += W.n) {
    const int pr = (p0 + W.t) / T;
    float sum = 0.f;
    if (pr < pairs) {
      const int i = pr / Kn, j = pr - i * Kn;
      const float4* q4 = reinterpret_cast<const float4*>(qs + i * hd);
      const float4* k4 = reinterpret_cast<const float4*>(ks + j * hd);
      for (int c = gl; c < cpr; c += T) {
        const float4 a = q4[c], k = k4[c];
        sum += a.x * k.x + a.y * k.y + a.z * k.z + a.w * k.w;
      }
    }
    for (int off = T >> 1; off > 0; off >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, off);
    if (pr < pairs && gl == 0) {
      const int i = pr / Kn, j = pr - i * Kn;
      sc[pr] = (A.causal && j > i) ? -INFINITY : sum * A.scale;
    }
  }
  gsync(W);
  if (W.t < Sq) {
    float* row = sc + W.t * Kn;
    float mx = -INFINITY;
    for (int j = 0; j < Kn; ++j) mx = fmaxf(mx, row[j]);
    float sum = 0.f;
    for (int j = 0; j < Kn; ++j) { const float e = __expf(row[j] - mx); row[j] = e; sum += e; }
    const float inv = 1.f / sum;
    for (int j = 0; j < Kn; ++j) row[j] *= inv;
  }
  gsync(W);
  // out[i, 4c..4c+3] = sum_j p[i, j] v[j, 4c..4c+3] -> four consecutive fp16 of the tiled output
  for (int e = W.t; e < Sq * cpr; e += W.n) {
    const int i = e / cpr, c = e - i * cpr;
    float4 o = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int j = 0; j < Kn; ++j) {
      const float pj = sc[i * Kn + j];
      const float4 v = reinterpret_cast<const float4*>(vs + j * hd)[c];
      o.x += pj * v.x; o.y += pj * v.y; o.z += pj * v.z; o.w += pj * v.w;
    }
    uint2 pk;
    pk.x = pack_half2(o.x, o.y);
    pk.y = pack_half2(o.z, o.w);
    *reinterpret_cast<uint2*>(A.out + tidx(A.outR, b * Sq + i, h * hd + 4 * c)) = pk;
  }
  gsync(W);
}

// An attention phase: its (task, request, head) items spread over the CTAs, one at a time.
__device__ __noinline__ void attn_phase(const Plan& P, const Phase& ph, const AttnTask* at, Smem& S, const Grp& W) {
  for (int t = blockIdx.x; t < ph.ntiles; t += P.G) {
    int jx = 0, rem = t;
    for (; jx < ph.njobs; ++jx) {
      const AttnTask& A = at[jx];
      const int n = A.B * A.heads;
      if (rem < n) break;
      rem -= n;
    }
    if (jx >= ph.njobs) break;
    const AttnTask& A = at[jx];
    attn_task(A, rem / A.heads, rem % A.heads, S, W);
  }
}

// ------------------------------------------------------------------------------------------
CFB_DEV bool better(float v, int i, float w, int j) { return v > w || (v == w && i < j); }

// static-index insertion into a descending top list (stays in registers)
CFB_DEV void top_insert(HeadState& H, int K, float v, int id) {
#pragma unroll
  for (int i = 0; i < kTopMax; ++i) {
    if (i < K && better(v, id, H.tv[i], H.ti[i])) {
      const float tv = H.tv[i]; const int ti = H.ti[i];
      H.tv[i] = v; H.ti[i] = id; v = tv; id = ti;
    }
  }
}

CFB_DEV void head_reset(HeadState& H) {
  H.m = -INFINITY; H.s = 0.f;
#pragma unroll
  for (int i = 0; i < kTopMax; ++i) { H.tv[i] = -INFINITY; H.ti[i] = 0x7fffffff; }
}

// entry j of a sorted top list (-inf past its end), without indexing registers at run time
CFB_DEV void list_at(const HeadState& H, int j, float& v, int& id) {
  v = -INFINITY; id = 0x7fffffff;
#pragma unroll
  for (int i = 0; i < kTopMax; ++i) if (i == j) { v = H.tv[i]; id = H.ti[i]; }
}

// better (value, id, owner) across the lanes of aligned groups of `width` lanes (xor tree)
CFB_DEV void argmax_lanes(float& v, int& id, int& own, int width) {
  for (int off = 1; off < width; off <<= 1) {
    const float vo = __shfl_xor_sync(0xffffffffu, v, off);
    const int io = __shfl_xor_sync(0xffffffffu, id, off), oo = __shfl_xor_sync(0xffffffffu, own, off);
    if (better(vo, io, v, id) || (vo == v && io == id && oo < own)) { v = vo; id = io; own = oo; }
  }
}

CFB_DEV void lse_merge(float& m, float& s, float mb, float sb) {
  const float M = fmaxf(m, mb);
  s = (M == -INFINITY) ? 0.f : s * __expf(m - M) + sb * __expf(mb - M);
  m = M;
}

// (max, sumexp) across aligned groups of `width` lanes; the lower lane is the left operand
CFB_DEV void lse_lanes(float& m, float& s, int width) {
  const int lane = threadIdx.x & 31;
  for (int off = 1; off < width; off <<= 1) {
    const float mo = __shfl_xor_sync(0xffffffffu, m, off), so = __shfl_xor_sync(0xffffffffu, s, off);
    if (lane & off) { float m1 = mo, s1 = so; lse_merge(m1, s1, m, s); m = m1; s = s1; }
    else lse_merge(m, s, mo, so);
  }
}

// ------------------------------------------------------------------------------------------
// the fused epilogue of one completed 64-feature tile (S.red holds its [feature][row] sums);
// per-row work loads its global operands in unrolled groups of 8 so the loads overlap
CFB_DEV void tile_epilogue(const Plan& P, const Job& J, int tile, Smem& S, HeadState& H, const Grp& E) {
  const int rows = J.rows;
  const int col0 = tile * kTileRows;
  switch (J.ekind) {
    case EK_STORE:
    case EK_STORE16:
    case EK_GELU16: {
      // the job's fields in registers (a store through a generic pointer could alias the cached
      // job in shared memory), and four elements' operands loaded before the first store
      const int ek = J.ekind, nout = J.nout, oR = J.oR, total = kTileRows * rows;
      const size_t ldo = (size_t)J.ldo;
      float* const out32 = J.out32;
      __half* const out16 = J.out16;
      constexpr int kU = 4;
      for (int e0 = E.t; e0 < total; e0 += kU * E.n) {
        float v[kU];
        int rr[kU], cc[kU];
        bool ok[kU];
#pragma unroll
        for (int u = 0; u < kU; ++u) {
          const int e = e0 + u * E.n;
          const int r = e / kTileRows, f = e - r * kTileRows;      // consecutive threads: columns
          rr[u] = r; cc[u] = col0 + f;
          ok[u] = e < total && cc[u] < nout;
          v[u] = ok[u] ? epi_val(S, f, r) : 0.f;
        }
#pragma unroll
        for (int u = 0; u < kU; ++u) {
          if (!ok[u]) continue;
          if (ek == EK_STORE) out32[(size_t)rr[u] * ldo + cc[u]] = v[u];
          else if (ek == EK_STORE16) out16[(size_t)rr[u] * ldo + cc[u]] = __float2half_rn(v[u]);   // row-major
          else out16[tidx(oR, rr[u], cc[u])] = __float2half_rn(gelu_erf(v[u]));
        }
      }
      break;
    }
    case EK_HEADIN: {
      for (int e = E.t; e < kTileRows * rows; e += E.n) {
        const int r = e / kTileRows, f = e - r * kTileRows;
        const int col = col0 + f;
        const int b = r / J.wrows;
        J.out16[tidx(J.oR, r, col)] =
            __float2half_rn(epi_val(S, f, r) + P.pred[((size_t)b * P.DL + J.step) * P.D + col]);
      }
      break;
    }
    case EK_RESID:
    case EK_PATHH: {
      const RowMap M = row_map(rows, E.t, E.n);
      float m = 0.f, M2 = 0.f;
      int ng = 0;
      if (M.r < rows) {
        for (int f0 = M.q * M.nf; f0 < (M.q + 1) * M.nf; f0 += 8) {
          float add[8];
          if (J.ekind == EK_RESID) {
            // 8 consecutive fp32 columns from a multiple of 8: two 16-byte loads
            const float4* a4 = reinterpret_cast<const float4*>(J.out32 + (size_t)M.r * J.ldo + col0 + f0);
            const float4 a = a4[0], c = a4[1];
            add[0] = a.x; add[1] = a.y; add[2] = a.z; add[3] = a.w;
            add[4] = c.x; add[5] = c.y; add[6] = c.z; add[7] = c.w;
          } else {
#pragma unroll
            for (int i = 0; i < 8; ++i) add[i] = 0.f;
            const int64_t* lp = P.lastp + ((size_t)(M.r / J.wrows) * P.Wmax + M.r % J.wrows) * J.order;
            for (int j = 0; j < J.nlive; ++j)
              if (lp[j] >= 0) {
#pragma unroll
                for (int i = 0; i < 8; ++i) add[i] += J.p0[(size_t)j * J.D + col0 + f0 + i];
              }
          }
          float v[8];
#pragma unroll
          for (int i = 0; i < 8; ++i) v[i] = epi_val(S, f0 + i, M.r) + add[i];
          if (J.ekind == EK_RESID) {
            float4* o32 = reinterpret_cast<float4*>(J.out32 + (size_t)M.r * J.ldo + col0 + f0);
            o32[0] = make_float4(v[0], v[1], v[2], v[3]);
            o32[1] = make_float4(v[4], v[5], v[6], v[7]);
          }
          // 8 consecutive columns from a multiple of 8 are 16 contiguous bytes of the tiled layout
          *reinterpret_cast<uint4*>(J.out16 + tidx(J.oR, M.r, col0 + f0)) =
              make_uint4(pack_half2(v[0], v[1]), pack_half2(v[2], v[3]), pack_half2(v[4], v[5]), pack_half2(v[6], v[7]));
          float mb, qb;
          stats8(v, mb, qb);
          stats8_add(m, M2, ng++, mb, qb);
        }
      }
      eq_group(m, M2, (float)M.nf, M.sl);
      if (M.q == 0 && M.r < rows) J.ostats[(size_t)M.r * J.onparts + tile] = make_float2(m, M2);
      break;
    }
    case EK_EULER: {
      const RowMap M = row_map(rows, E.t, E.n);
      const int b = M.r / P.chunk, c = M.r - b * P.chunk;
      const int pos = P.ex[J.e_idx].start + c;
      const int nx = (J.step + 1) & 1;
      const bool live = M.r < rows;
      const bool next = !J.last_step;
      const int f0 = M.q * M.nf, ne = P.n_experts;
      const float dt = J.dt;
      // per expert that sees this position: the running statistics of its next-step input row
      float m[kMaxExperts], M2[kMaxExperts];
#pragma unroll
      for (int e = 0; e < kMaxExperts; ++e) { m[e] = 0.f; M2[e] = 0.f; }
      if (live) {
        int ng = 0;
        for (int f = f0; f < f0 + M.nf; f += 8, ++ng) {
          // z <- z + dt * v on this tile's columns of the chunk rows (reference tree_flow.py:229-235);
          // 8 consecutive fp32 columns from a multiple of 8 move as two 16-byte accesses
          float4* z4 = reinterpret_cast<float4*>(P.pred + ((size_t)b * P.DL + pos) * P.D + col0 + f);
          const float4 za = z4[0], zb = z4[1];
          float z[8] = {za.x, za.y, za.z, za.w, zb.x, zb.y, zb.z, zb.w};
#pragma unroll
          for (int i = 0; i < 8; ++i) z[i] += dt * epi_val(S, f + i, M.r);
          z4[0] = make_float4(z[0], z[1], z[2], z[3]);
          z4[1] = make_float4(z[4], z[5], z[6], z[7]);
          if (!next) continue;
          // next step's inputs of every expert that sees this position: z + pos (+ time on its
          // chunk), from the z just computed
#pragma unroll
          for (int e = 0; e < kMaxExperts; ++e) {
            if (e >= ne) break;
            const ExpertRT& X = P.ex[e];
            if (pos >= X.S) continue;
            const bool cur = pos >= X.start;
            const int xrow = b * X.S + pos;
            const float4* pe4 = reinterpret_cast<const float4*>(X.pos + (size_t)pos * P.D + col0 + f);
            const float4* te4 = reinterpret_cast<const float4*>(X.temb + (size_t)(J.step + 1) * P.D + col0 + f);
            const float4 pa = pe4[0], pb = pe4[1];
            float4 ta = make_float4(0.f, 0.f, 0.f, 0.f), tb = ta;
            if (cur) { ta = te4[0]; tb = te4[1]; }
            const float pe[8] = {pa.x, pa.y, pa.z, pa.w, pb.x, pb.y, pb.z, pb.w};
            const float te[8] = {ta.x, ta.y, ta.z, ta.w, tb.x, tb.y, tb.z, tb.w};
            float xv[8];
#pragma unroll
            for (int i = 0; i < 8; ++i) xv[i] = z[i] + pe[i] + (cur ? te[i] : 0.f);
            float4* x4 = reinterpret_cast<float4*>(X.x32[nx] + (size_t)xrow * P.D + col0 + f);
            x4[0] = make_float4(xv[0], xv[1], xv[2], xv[3]);
            x4[1] = make_float4(xv[4], xv[5], xv[6], xv[7]);
            // 8 consecutive columns from a multiple of 8 are 16 contiguous bytes of the tiled layout
            *reinterpret_cast<uint4*>(X.x16[nx] + tidx(P.B * X.S, xrow, col0 + f)) =
                make_uint4(pack_half2(xv[0], xv[1]), pack_half2(xv[2], xv[3]), pack_half2(xv[4], xv[5]),
                           pack_half2(xv[6], xv[7]));
            float mb, qb;
            stats8(xv, mb, qb);
            stats8_add(m[e], M2[e], ng, mb, qb);
          }
        }
      }
      if (!next) break;
#pragma unroll
      for (int e = 0; e < kMaxExperts; ++e) {
        if (e >= ne) break;
        const ExpertRT& X = P.ex[e];
        const bool has = live && pos < X.S;
        eq_group(m[e], M2[e], (float)M.nf, M.sl);
        if (M.q == 0 && has) X.xstat[nx][((size_t)b * X.S + pos) * (P.D / kStatCols) + tile] = make_float2(m[e], M2[e]);
      }
      break;
    }
    case EK_HEAD: {
      const RowMap M = head_map(rows, E.t, E.n);
      if (M.r < rows) {
        const int rq = J.cmask ? M.r / J.wrows : 0;
        for (int f = M.q * M.nf; f < (M.q + 1) * M.nf; ++f) {
          const int j = col0 + f;
          if (j >= J.R) break;
          const float v = S.red[f * S.rp + M.r];
          if (J.logits) J.logits[(size_t)M.r * J.R + j] = v;
          if (J.cmask && j / J.cmask != rq) continue;
          if (v > H.m) { H.s = H.s * __expf(H.m - v) + 1.f; H.m = v; }
          else H.s += __expf(v - H.m);
          // pass B: a candidate column; the candidates of a request are in ascending shortlist
          // order, so ties still go to the lower shortlist id (mapped when the lists are published)
          top_insert(H, J.topb, v, j + J.rowoff);
        }
      }
      break;
    }
  }
  gsync(E);
}

// ------------------------------------------------------------------------------------------
// While the MMA warps still work on a tile: pull the global operands of its epilogue (the rows it
// adds to or updates, two 128-byte lines per row of 64 fp32 columns) into L1.
CFB_DEV void prefetch_l1(const void* p) { asm volatile("prefetch.global.L1 [%0];" :: "l"(p)); }
CFB_DEV void epi_prefetch(const Plan& P, const Job& J, int tile, const Grp& E) {
  const int col0 = tile * kTileRows;
  for (int e = E.t; e < 2 * J.rows; e += E.n) {
    const int r = e >> 1, c = col0 + 32 * (e & 1);
    const float* p = nullptr;
    if (J.ekind == EK_RESID) {
      p = J.out32 + (size_t)r * J.ldo + c;
    } else if (J.ekind == EK_HEADIN) {
      p = P.pred + ((size_t)(r / J.wrows) * P.DL + J.step) * P.D + c;
    } else if (J.ekind == EK_EULER) {
      const int b = r / P.chunk, pos = P.ex[J.e_idx].start + (r - b * P.chunk);
      p = P.pred + ((size_t)b * P.DL + pos) * P.D + c;
    }
    if (p) prefetch_l1(p);
  }
}

// Epilogue side of one tile: take the MMA warps' partials from slot buffer `b`, reduce them in a
// fixed order, release the slot, then finish the tile directly or through the stream-K fixup.
constexpr int kFixBatch = 3;   // contributors whose partials one fixup step loads at once
// E: the threads that finish the tile (the epilogue warps, or in a wide-epilogue phase those and
// worker warps 1..7); `reader`: this thread is an epilogue warp's, which alone wait for and read
// the accumulator (tensor-memory lane quarters are per warp).
template <class WaitClock>
CFB_DEV void epi_tile(const Plan& P, const Job& J, int tile, bool complete, long long U,
                      long long ug_first, uint32_t& tseq, Smem& S,
                      HeadState& H, const Grp& E, bool reader, WaitClock& wc) {
  const int rows = J.rows;
  const int b = tseq % S.nbuf;
  epi_prefetch(P, J, tile, E);
  {   // this tile's bias and LayerNorm column sums, one load per thread, before the partials
      // are ready (the previous tile's epilogue has finished with these arrays)
    const int col0 = tile * kTileRows;
    if (E.t < kTileRows) {
      const int col = col0 + E.t;
      S.tbias[E.t] = (J.bias && col < J.nout) ? J.bias[col] : 0.f;
    } else if (E.t < 2 * kTileRows) {
      const int col = col0 + E.t - kTileRows;
      S.tcsum[E.t - kTileRows] = (J.colsum && col < J.nout) ? J.colsum[col] : 0.f;
    }
  }
  const bool ident = J.goff == 0 && (J.gin >= rows || J.gstride == J.gin);
  if (reader) {
  const unsigned long long w0 = wc.now();
  if (!mbar_wait(&S.accf[b], (tseq / S.nbuf) & 1, P.err)) set_err(P, DEV_TIMEOUT_SLOT);
  if (wc.on) { wc.part = wc.now(); wc.slot += wc.part - w0; wc.atom = wc.fix = 0; }
  tc_fence_after();
  // The accumulator of an M = 64 MMA: feature f sits in TMEM lane 32 (f / 16) + f % 16, the
  // value for slot row c in column c. Each epilogue warp reads its lane quarter (warp % 4), 16
  // columns at a time; output row r is slot row src_row(r) (the identity but for gathered rows).
  {
    const int q = (threadIdx.x >> 5) & 3, lane = threadIdx.x & 31;
    const int f = 16 * q + (lane & 15);
    const int ncol = ident ? rows : (J.xcopy + 7) & ~7;
    const uint32_t ta = S.tmem + ((uint32_t)(32 * q) << 16) + (uint32_t)(b * kAccCols);
    for (int c0 = 0; c0 < ncol; c0 += 16) {
      float v[16];
      tmem_ld16(ta + (uint32_t)c0, v);
      if (lane < 16) {
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          if (c0 + i >= ncol) break;
          if (ident) S.red[f * S.rp + c0 + i] = v[i];
          else S.slots[f * (kAccCols + 1) + c0 + i] = v[i];
        }
      }
    }
  }
  tc_fence_before();
  }
  gsync(E);
  if (E.t == 0) mbar_arrive(&S.acce[b]);
  if (!ident) {
    for (int e = E.t; e < kTileRows * rows; e += E.n) {
      const int f = e / rows, r = e - f * rows;
      S.red[f * S.rp + r] = S.slots[f * (kAccCols + 1) + src_row(J, r)];
    }
    gsync(E);
  }
  ++tseq;
  if (!complete) {
    // A tile split across CTAs (stream-K). Its owner is the CTA whose range holds the tile's
    // first unit; that unit range ends the owner's own range, so the owner reaches the tile last
    // and finishes it. Every other contributor holds the tile's later units at the START of its
    // range: it publishes its partial there (at most one per CTA and phase) and counts itself in.
    // The owner waits (bounded) for the count, then adds the partials in k order to its own.
    // Nobody else waits on anything, so the waits cannot form a cycle.
    const int c = blockIdx.x;
    unsigned* cnt = P.tilecnt + J.tile_base + tile;
    if (cta_start(U, P.G, c) > ug_first) {
      float* mine = P.gpart + (size_t)c * (kTileRows * kRowsMax);
      for (int e = E.t; e < kTileRows * rows; e += E.n) {
        const int f = e / rows, r = e - f * rows;
        __stcg(mine + f * kRowsMax + r, S.red[f * S.rp + r]);
      }
      gsync(E);
      // the barrier orders every thread's partial stores before thread 0's release count
      if (E.t == 0) {
        atom_add_release(cnt, 1u);
        if (wc.on) wc.atom = wc.now();
      }
      return;
    }
    // owner: list the other contributors (CTA ids, in k order) in the epilogue scratch
    int* clist = reinterpret_cast<int*>(S.scratch);
    if (E.t == 0) {
      const long long ug_last = ug_first + J.nkc - 1;
      int n = 0;
      for (int cc = next_contributor(c, U, P.G); cc < P.G && cta_start(U, P.G, cc) <= ug_last;
           cc = next_contributor(cc, U, P.G))
        clist[1 + n++] = cc;
      clist[0] = n;
      const unsigned want = (unsigned)n;
      const unsigned long long t0 = globaltimer();
      for (unsigned it = 1; ld_acquire(cnt) < want; ++it) {
        if (it % kPollsPerCheck) continue;
        if (ld_volatile_int(P.err) != 0) break;
        if (globaltimer() - t0 > kWaitBudgetNs) { set_err(P, DEV_TIMEOUT_FIXUP); break; }
      }
      *cnt = 0u;               // reused by the same tile index of the next split phase
      if (wc.on) wc.atom = wc.now();
    }
    gsync(E);
    const int ncontrib = clist[0];
    const int total = kTileRows * rows;
    for (int e0 = E.t; e0 < total; e0 += 8 * E.n) {
      int off[8];
      float acc[8];
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        const int e = e0 + k * E.n;
        const int f = e / rows, r = e - f * rows;
        off[k] = e < total ? f * kRowsMax + r : -1;
        acc[k] = e < total ? S.red[f * S.rp + r] : 0.f;
      }
      // the partials are added in k order, but the loads of kFixBatch contributors are all
      // issued before the first add, so their L2 round trips overlap instead of queueing
      for (int i0 = 0; i0 < ncontrib; i0 += kFixBatch) {
        float v[kFixBatch][8];
#pragma unroll
        for (int j = 0; j < kFixBatch; ++j) {
          const bool on = i0 + j < ncontrib;
          const float* part = P.gpart + (size_t)clist[1 + (on ? i0 + j : i0)] * (kTileRows * kRowsMax);
#pragma unroll
          for (int k = 0; k < 8; ++k) v[j][k] = (on && off[k] >= 0) ? __ldcg(part + off[k]) : 0.f;
        }
#pragma unroll
        for (int j = 0; j < kFixBatch; ++j) {
#pragma unroll
          for (int k = 0; k < 8; ++k) acc[k] += v[j][k];
        }
      }
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        const int e = e0 + k * E.n;
        if (e < total) { const int f = e / rows, r = e - f * rows; S.red[f * S.rp + r] = acc[k]; }
      }
    }
    gsync(E);
    if (wc.on) wc.fix = wc.now();
  }
  tile_epilogue(P, J, tile, S, H, E);
  if (wc.on) wc.tdone = wc.now();
}

// ------------------------------------------------------------------------------------------
// The units of a phase for this CTA: one contiguous range of the phase's linear unit space,
// walked job by job. The weight producer, the activation producer, the MMA warps and the
// epilogue warps all walk exactly this sequence, so ring slot i always holds the i-th unit and
// slot buffer j the j-th tile.
struct UnitRange { long long u0, u1; };
// first unit of the phase's t-th tile (tiles are numbered across the phase's jobs)
CFB_DEV long long tile_unit(const Phase& ph, const Job* jt, long long t) {
  if (t >= ph.ntiles) return ph.nunits;
  for (int jx = ph.njobs - 1; jx >= 0; --jx) {
    const Job& J = jt[jx];
    if (t >= J.tile_base) return J.unit_base + (t - J.tile_base) * J.nkc;
  }
  return 0;
}
CFB_DEV UnitRange cta_units(const Plan& P, const Phase& ph, const Job* jt) {
  if (ph.whole) {
    const long long T = ph.ntiles;
    return {tile_unit(ph, jt, cta_start(T, P.G, blockIdx.x)), tile_unit(ph, jt, cta_start(T, P.G, blockIdx.x + 1))};
  }
  const long long U = ph.nunits;
  return {cta_start(U, P.G, blockIdx.x), cta_start(U, P.G, blockIdx.x + 1)};
}
CFB_DEV bool job_slice(const Job& J, const UnitRange& cu, int& ju0, int& ju1) {
  const long long jb = J.unit_base, je = jb + (long long)J.Mt * J.nkc;
  const long long a = max(cu.u0, jb), b = min(cu.u1, je);
  if (a >= b) return false;
  ju0 = (int)(a - jb); ju1 = (int)(b - jb);
  return true;
}

// The MMA warp (kMmaIssueWarp; all 32 lanes walk this loop converged, so every operand below is
// warp-uniform, and one elected lane issues): for each of this CTA's units, once its ring stage is
// full, D[tmem] (+)= W_unit X_unit^T over the unit's k blocks with tcgen05.mma (M = 64 features,
// N = the job's slot rows padded to 8, K = 16 per instruction, both operands K-major with the
// 128-byte swizzle, straight from the ring stage), then tcgen05.commit returns the stage to the
// producers once those MMAs have read it. The last unit of a tile (or of this CTA's share of it)
// commits the accumulator to the epilogue; a tile's first MMA overwrites the accumulator, after
// the epilogue has released that TMEM buffer. Nothing here holds accumulators in registers.
template <class WaitClock>
CFB_DEV void tc_phase(const Plan& P, const Phase& ph, const Job* jt, uint32_t& ci, uint32_t& tseq, Smem& S,
                      WaitClock& wc) {
  const UnitRange cu = cta_units(P, ph, jt);
  const int* err = P.err;
  // everything the unit loop touches is held in registers: the asm statements below clobber
  // memory, so a field read through S or a Job reference would be reloaded at every MMA
  const int nst = S.nstages, nbuf = S.nbuf;
  const uint32_t ring = smem_u32(S.ring), sbytes = (uint32_t)S.stage_bytes, xhalf = (uint32_t)S.xhalf;
  const uint32_t full0 = smem_u32(S.full), empty0 = smem_u32(S.empty);
  const uint32_t accf0 = smem_u32(S.accf), acce0 = smem_u32(S.acce), tmem = S.tmem;
  const bool prof = wc.on;
  for (int jx = 0; jx < ph.njobs; ++jx) {
    const Job& J = jt[jx];
    int ju0, ju1;
    if (!job_slice(J, cu, ju0, ju1)) continue;
    const int nkc = J.nkc, Kt = J.Kt;
    const uint32_t idesc = tc_idesc(kTileRows, (J.xcopy + 7) & ~7);
    int stage = (int)(ci % (uint32_t)nst);
    uint32_t par = (ci / (uint32_t)nst) & 1u;
    int slot = (int)(tseq % (uint32_t)nbuf);
    uint32_t spar = (tseq / (uint32_t)nbuf) & 1u;
    int kc = ju0 % nkc;
    int nkb_left = Kt - kc * kUnitK;   // k blocks of the tile from this unit on
    bool fresh = true;                 // the next unit starts a tile (of this CTA's share)
    for (int ju = ju0; ju < ju1; ++ju) {
      const int nkb = min(kUnitK, nkb_left);
      if (fresh) {
        const unsigned long long w1 = prof ? globaltimer() : 0ull;
        if (!mbar_wait_a(acce0 + 8u * (uint32_t)slot, spar ^ 1u, err)) set_err(P, DEV_TIMEOUT_SLOT);
        if (prof) wc.slot += globaltimer() - w1;
        __syncwarp();
        tc_fence_after();   // the epilogue's reads of this accumulator come before the MMAs below
      }
      const unsigned long long w0 = prof ? globaltimer() : 0ull;
      if (!mbar_wait_a(full0 + 8u * (uint32_t)stage, par, err)) set_err(P, DEV_TIMEOUT_FULL);
      if (prof) {
        const unsigned long long w1 = globaltimer();
        wc.full += w1 - w0;
        if (wc.first == 0) wc.first = w1;
        wc.last = w1;
      }
      __syncwarp();
      const uint32_t ws = ring + (uint32_t)stage * sbytes, xs = ws + kUnitBytes;
      const uint32_t td = tmem + (uint32_t)(slot * kAccCols);
      const uint64_t a0 = sw128_desc(ws), b0 = sw128_desc(xs);
      const uint64_t a1 = sw128_desc(ws + kHalfBytes), b1 = sw128_desc(xs + xhalf);
      // k block kb sits in half kb / 4 at byte offset 32 (kb % 4): +2 in the descriptor's
      // 16-byte start-address field per k block
      if (nkb == kUnitK) {             // a whole unit: 8 MMAs and the stage's commit in one go
        tc_unit8_warp(td, a0, b0, a1, b1, idesc, fresh ? 0u : 1u, empty0 + 8u * (uint32_t)stage);
      } else {
        tc_mma_f16_warp(td, a0, b0, idesc, fresh ? 0u : 1u);
        for (int kb = 1; kb < nkb; ++kb) {
          const uint64_t o = (uint64_t)((kb & 3) * 2);
          tc_mma_f16_warp(td, (kb < 4 ? a0 : a1) + o, (kb < 4 ? b0 : b1) + o, idesc, 1u);
        }
        tc_commit_warp_a(empty0 + 8u * (uint32_t)stage);
      }
      fresh = false;
      if (++stage == nst) { stage = 0; par ^= 1u; }
      ++ci;
      nkb_left -= kUnitK;
      if (++kc == nkc || ju == ju1 - 1) {
        tc_commit_warp_a(accf0 + 8u * (uint32_t)slot);
        if (++slot == nbuf) { slot = 0; spar ^= 1u; }
        ++tseq;
        fresh = true;
        if (kc == nkc) { kc = 0; nkb_left = Kt; }
      }
    }
  }
}

// Epilogue warps: the same tiles in the same order.
template <class WaitClock>
CFB_DEV void epi_phase(const Plan& P, const Phase& ph, const Job* jt, uint32_t& tseq, Smem& S, HeadState& H,
                       const Grp& E, bool reader, WaitClock& wc) {
  const long long U = ph.nunits;
  const UnitRange cu = cta_units(P, ph, jt);
  for (int jx = 0; jx < ph.njobs; ++jx) {
    const Job& J = jt[jx];
    int ju0, ju1;
    if (!job_slice(J, cu, ju0, ju1)) continue;
    job_rowstats(J, S, E);
    if (wc.on) wc.rstat = wc.now();
    for (int tile = ju0 / J.nkc; tile <= (ju1 - 1) / J.nkc; ++tile) {
      const bool complete = (ju0 <= tile * J.nkc) && (ju1 >= (tile + 1) * J.nkc);
      epi_tile(P, J, tile, complete, U, (long long)J.unit_base + (long long)tile * J.nkc, tseq, S, H, E, reader, wc);
    }
  }
}

// Weight producer (one thread): stream this CTA's packed weight units of every GEMM phase into
// the ring with cp.async.bulk, running ahead of the consumers across phase boundaries. (An L2
// prefetch running further ahead than the ring was measured and not kept: with 8 to 32 units
// per CTA ahead, DRAM reads grew by up to 1.75x, the prefetched lines being evicted before use,
// and the 4B draft slowed from 5.35 to 5.8-6.8 ms.)
CFB_DEV void weight_producer(const Plan& P, Smem& S, int p0, int p1) {
  uint32_t pi = 0;
  int stage = 0;
  uint32_t par = 1u;                 // a fresh mbarrier's previous phase counts as complete
  bool ok = true;
  const int nst = S.nstages;
  const int* err = P.err;
  const bool prof = P.prof != nullptr;
  for (int p = p0; p < p1 && ok; ++p) {
    const Phase& ph = P.phases[p];
    if (ph.kind != PK_GEMM) continue;
    if (ph.last == kWeightsWritten) {
      // these weights are written by an earlier phase of this launch (the two-pass head's
      // gathered candidate rows): stream them only once the workers have entered this phase
      const unsigned long long t0 = globaltimer();
      for (unsigned it = 1; *S.phase_ready < p; ++it) {
        if (it % kPollsPerCheck) continue;
        if (ld_volatile_int(P.err) != 0) { ok = false; break; }
        if (globaltimer() - t0 > kWaitBudgetNs) { set_err(P, DEV_TIMEOUT_SLOT); ok = false; break; }
      }
      if (!ok) break;
      __threadfence();
      fence_proxy_async_global();
    }
    unsigned long long waited = 0;
    const Job* jt = P.jobs + ph.job0;
    const UnitRange cu = cta_units(P, ph, jt);
    for (int jx = 0; jx < ph.njobs && ok; ++jx) {
      const Job& J = jt[jx];
      int ju0, ju1;
      if (!job_slice(J, cu, ju0, ju1)) continue;
      const int nkc = J.nkc, Kt = J.Kt;
      const uint8_t* wbase = reinterpret_cast<const uint8_t*>(J.w);
      const size_t tile_bytes = (size_t)J.Kstride * 4 * kBlockBytes;
      int tile = ju0 / nkc, kc = ju0 - tile * nkc;
      for (int ju = ju0; ju < ju1; ++ju) {
        const int nkb = min(kUnitK, Kt - kc * kUnitK);
        const uint8_t* src = wbase + (size_t)tile * tile_bytes + (size_t)kc * kUnitBytes;
        // whole [64 x 64] halves: a unit of at most 64 k streams one
        const uint32_t bytes = nkb > 4 ? (uint32_t)kUnitBytes : (uint32_t)kHalfBytes;
        const unsigned long long w0 = prof ? globaltimer() : 0ull;
        if (!mbar_wait(&S.empty[stage], par, err)) {
          set_err(P, DEV_TIMEOUT_EMPTY); ok = false; break;
        }
        if (prof) waited += globaltimer() - w0;
        mbar_arrive_expect_tx(&S.full[stage], bytes);
        bulk_g2s(S.ring + (size_t)stage * S.stage_bytes, src, bytes, &S.full[stage]);
        ++pi;
        if (++stage == nst) { stage = 0; par ^= 1u; }
        if (++kc == nkc) { kc = 0; ++tile; }
      }
    }
    if (P.prof) {
      P.prof[((size_t)p * P.G + blockIdx.x) * kProfSlots + 8] = waited;
      P.prof[((size_t)p * P.G + blockIdx.x) * kProfSlots + 9] = globaltimer();
    }
  }
  // every issued copy must land before this CTA may exit (copies complete on their own)
  const uint32_t first = pi > (uint32_t)S.nstages ? pi - S.nstages : 0u;
  for (uint32_t i = first; i < pi; ++i) mbar_wait(&S.full[i % S.nstages], (i / S.nstages) & 1);
}

// Activation producer (one thread): once the grid barrier in front of a phase has passed, copy
// each unit's activation rows (its 128 columns: two 64-column slices of the tiled source, each
// one contiguous block) into the unit's ring slot with 1-D bulk copies that complete on the
// slot's full barrier (the same barrier the weight producer's copy completes on). A unit of at
// most 64 k takes one slice.
CFB_DEV void x_unit(const Job& J, int ju, uint8_t* xs, uint32_t xhalf, uint64_t* full) {
  const int kc = ju % J.nkc;
  const int nh = J.Kt - kc * kUnitK > 4 ? 2 : 1;
  const uint32_t bytes = (uint32_t)J.xcopy * 128u;
  mbar_arrive_expect_tx(full, bytes * (uint32_t)nh);
  for (int h = 0; h < nh; ++h) bulk_g2s(xs + (size_t)h * xhalf, J.x + (size_t)(2 * kc + h) * J.xR * 64, bytes, full);
}

// The descriptor cache slot of phase p (one thread): the phase record, then, for a GEMM phase of
// at most kJobCache jobs, its jobs, 16 loads in flight at a time; published through
// S.desc_ready.
CFB_DEV void desc_fill(const Plan& P, Smem& S, int p) {
  uint8_t* slot = S.desc + (size_t)(p % kDescBufs) * (kPhaseSlot + kJobCache * sizeof(Job));
  constexpr int kPhInts = (int)(sizeof(Phase) / sizeof(int));
  const int* ps = reinterpret_cast<const int*>(P.phases + p);
  int v[kPhInts];
#pragma unroll
  for (int i = 0; i < kPhInts; ++i) v[i] = __ldcg(ps + i);
#pragma unroll
  for (int i = 0; i < kPhInts; ++i) reinterpret_cast<int*>(slot)[i] = v[i];
  const int kind = v[0], job0 = v[1], njobs = v[2];
  const bool gemm = kind == PK_GEMM && njobs <= kJobCache, attn = kind == PK_ATTN && njobs <= kAttnCache;
  if (gemm || attn) {
    const int n16 = gemm ? njobs * (int)(sizeof(Job) / 16) : njobs * (int)(sizeof(AttnTask) / 16);
    const uint4* src = gemm ? reinterpret_cast<const uint4*>(P.jobs + job0) : reinterpret_cast<const uint4*>(P.attn + job0);
    uint4* dst = reinterpret_cast<uint4*>(slot + kPhaseSlot);
    for (int i0 = 0; i0 < n16; i0 += 16) {
      uint4 t[16];
#pragma unroll
      for (int i = 0; i < 16; ++i)
        if (i0 + i < n16) t[i] = __ldcg(src + i0 + i);
#pragma unroll
      for (int i = 0; i < 16; ++i)
        if (i0 + i < n16) dst[i0 + i] = t[i];
    }
  }
  __threadfence_block();
  *S.desc_ready = p;
}

// The jobs of cached phase p (the descriptor cache, or the global table beyond kJobCache jobs).
CFB_DEV const Job* phase_jobs(const Plan& P, const Smem& S, const Phase& ph, int p) {
  return ph.njobs <= kJobCache ? S.djobs(p) : P.jobs + ph.job0;
}
// The attention tasks of cached phase p.
CFB_DEV const AttnTask* phase_tasks(const Plan& P, const Smem& S, const Phase& ph, int p) {
  return ph.njobs <= kAttnCache ? reinterpret_cast<const AttnTask*>(S.djobs(p)) : P.attn + ph.job0;
}

// Activation producer (one thread): copies the activation rows of this CTA's units, and fills
// the descriptor cache a phase ahead of the workers. At the top of iteration p it fills phase
// p + 1's slot, which last held phase p - 2: the workers are past it, since iteration p - 1
// waited for them to enter phase p - 1.
CFB_DEV void x_producer(const Plan& P, Smem& S, int p0, int p1) {
  uint32_t xi = 0;            // units issued
  int xstage = 0;
  uint32_t xpar = 1u;         // a fresh mbarrier's previous phase counts as complete
  bool ok = true;
  desc_fill(P, S, p0);
  for (int p = p0; p < p1 && ok; ++p) {
    if (p + 1 < p1) desc_fill(P, S, p + 1);
    // Wait for the grid barrier in front of phase p. This thread polls the barrier counter itself
    // with acquire loads, which makes every CTA's writes of phase p - 1 visible to it, as they are
    // to the workers; a gpu-scope fence after the workers' shared-memory flag instead measured
    // about 0.9 us a phase. If this CTA's workers are already past the barrier (phase_ready; the
    // counter is reset once every CTA has left the launch), their flag is taken, with the fence.
    bool need_fence = p == p0;
    {
      const unsigned target = (unsigned)(p - p0) * (unsigned)P.G;
      const unsigned long long t0 = globaltimer();
      for (unsigned it = 1;; ++it) {
        if (p == p0) {
          if (*S.phase_ready >= p) break;
        } else {
          const unsigned v = ld_acquire(P.bar);
          if (v & kBarErrBit) { ok = false; break; }
          if (v >= target) break;
          if (*S.phase_ready >= p) { need_fence = true; break; }
        }
        if (it % kPollsPerCheck) continue;
        if (ld_volatile_int(P.err) != 0) { ok = false; break; }
        if (globaltimer() - t0 > kWaitBudgetNs) { set_err(P, DEV_TIMEOUT_SLOT); ok = false; break; }
      }
    }
    const Phase& ph = S.dphase(p);
    if (!ok || ph.kind != PK_GEMM) continue;
    const Job* jt = phase_jobs(P, S, ph, p);
    const UnitRange cu = cta_units(P, ph, jt);
    if (cu.u0 >= cu.u1) continue;
    // the rows were written by other SMs with ordinary stores; order them before the copy
    // engine (async proxy) reads them
    if (need_fence) __threadfence();
    fence_proxy_async_global();
    for (int jx = 0; jx < ph.njobs && ok; ++jx) {
      const Job& J = jt[jx];
      int ju0, ju1;
      if (!job_slice(J, cu, ju0, ju1)) continue;
      for (int ju = ju0; ju < ju1; ++ju) {
        if (!mbar_wait(&S.empty[xstage], xpar, P.err)) {
          set_err(P, DEV_TIMEOUT_EMPTY); ok = false; break;
        }
        x_unit(J, ju, S.ring + (size_t)xstage * S.stage_bytes + kUnitBytes, (uint32_t)S.xhalf, &S.full[xstage]);
        ++xi;
        if (++xstage == S.nstages) { xstage = 0; xpar ^= 1u; }
      }
    }
    if (P.prof) P.prof[((size_t)p * P.G + blockIdx.x) * kProfSlots + 7] = globaltimer();
  }
  // every issued copy must land before this CTA may exit (copies complete on their own)
  const uint32_t first = xi > (uint32_t)S.nstages ? xi - S.nstages : 0u;
  for (uint32_t i = first; i < xi; ++i) mbar_wait(&S.full[i % S.nstages], (i / S.nstages) & 1);
}

// ------------------------------------------------------------------------------------------
// initial latent z0[b, pos, col] (reference TreeFlowDrafter.init_latents, tree_flow.py:150-161):
// given (noise drawn by the caller), the last context row, or last + (pos+1) * (last - previous)
CFB_DEV float z0_at(const Plan& P, int b, int pos, int col) {
  if (P.init_mode == CFB_INIT_GIVEN) return __half2float(P.z0[((size_t)b * P.DL + pos) * P.D + col]);
  const float last = __half2float(P.ctx[((size_t)b * P.C + P.C - 1) * P.D + col]);
  if (P.init_mode == CFB_INIT_REPEAT_LAST || P.C < 2) return last;
  const float prev = __half2float(P.ctx[((size_t)b * P.C + P.C - 2) * P.D + col]);
  return last + (float)(pos + 1) * (last - prev);
}

// Head-input side rows of path-GEMM rows [row0, row0 + nrows) of a depth with R rows and `fr`
// rows per request: the embedding rows of the last `nlive` path tokens side by side (zeros for
// an absent token) into the path GEMM's tiled activation, and markov w1[last token] into the
// head input's columns [D, D + rank) (reference tree_flow.py:434-450, markov_flow.py:72-74).
// `from_known0`: depth 1, whose only path token is the committed one.
__device__ __noinline__ void path_gather(const Plan& P, int fr, int R, int row0, int nrows, int nlive, bool from_known0,
                         long long t, long long nt) {
  const int D = P.D, order = P.order, rank = P.rank;
  const int cpe = D / 8;                         // 16-byte chunks per embedding row
  const int cpr = nlive * cpe + rank / 8;        // chunks per gathered row
  const long long total = (long long)nrows * cpr;
  constexpr int kBatch = 4;                      // chunks per thread with their loads in flight together
  for (long long it0 = t; it0 < total; it0 += kBatch * nt) {
    uint4 val[kBatch];
    __half* dst[kBatch];
#pragma unroll
    for (int u = 0; u < kBatch; ++u) {
      const long long it = it0 + u * nt;
      val[u] = make_uint4(0u, 0u, 0u, 0u);
      dst[u] = nullptr;
      if (it >= total) continue;
      const int i = (int)(it / cpr), q = (int)(it - (long long)i * cpr);
      const int row = row0 + i, b = row / fr, w = row - b * fr;
      const int64_t* lp = P.lastp + ((size_t)b * P.Wmax + w) * order;
      if (q < nlive * cpe) {
        const int j = q / cpe, c = q - j * cpe;
        const int64_t tok = from_known0 ? (j == 0 ? P.known0[b] : (int64_t)-1) : lp[j];
        if (tok >= 0 && tok < P.vocab) val[u] = *reinterpret_cast<const uint4*>(P.emb + (size_t)tok * D + c * 8);
        dst[u] = P.pg + tidx(R, row, j * D + c * 8);
      } else {
        const int c = q - nlive * cpe;
        const int64_t tok = from_known0 ? P.known0[b] : lp[0];
        if (tok >= 0 && tok < P.vocab) val[u] = *reinterpret_cast<const uint4*>(P.markov_w1 + (size_t)tok * rank + c * 8);
        dst[u] = P.xhead + tidx(R, row, D + c * 8);
      }
    }
#pragma unroll
    for (int u = 0; u < kBatch; ++u) if (dst[u]) *reinterpret_cast<uint4*>(dst[u]) = val[u];
  }
}

__device__ __noinline__ void prep_phase(const Plan& P, const Grp& W) {
  const long long gtid = (long long)blockIdx.x * W.n + W.t;
  const long long gthreads = (long long)P.G * W.n;
  for (long long i = gtid; i < P.ntilecnt; i += gthreads) P.tilecnt[i] = 0u;
  if (P.tp_m) {   // the two-pass head's radix histograms and per-CTA counts start at zero
    for (long long i = gtid; i < 4LL * P.B * 256; i += gthreads) P.thist[i] = 0u;
    for (long long i = gtid; i < 2LL * P.B * P.G; i += gthreads) P.tcnt[i] = 0;
  }
  if (P.mode == kModeVae) {
    // the input rows, tiled for the in-projection's activation copies; the residual stream
    // starts at the learned position rows (the in-projection adds to it)
    const int Din = P.vDin, D = P.D, M = P.B * P.vS;
    for (long long i = gtid; i < (long long)M * Din; i += gthreads) {
      const int r = (int)(i / Din), c = (int)(i % Din);
      const __half h = P.vin32 ? __float2half_rn(static_cast<const float*>(P.vin)[i]) : static_cast<const __half*>(P.vin)[i];
      P.vin16[tidx(M, r, c)] = h;
    }
    for (long long i = gtid; i < (long long)M * D; i += gthreads) {
      const int r = (int)(i / D), c = (int)(i % D);
      P.vx32[i] = P.vpos[(size_t)(r % P.vS) * D + c];
    }
    return;
  }
  const bool flow = (P.mode == CFB_MODE_FLOW || P.mode == CFB_MODE_CHAIN || P.mode == CFB_MODE_TREE);
  const int D = P.D, nparts = D / kStatCols;
  if (flow) {
    const long long nz = (long long)P.B * P.DL * D;
    for (long long i = gtid; i < nz; i += gthreads)
      P.pred[i] = z0_at(P, (int)(i / ((long long)P.DL * D)), (int)((i / D) % P.DL), (int)(i % D));
    // step-0 inputs of every expert: z0 + position embedding (+ time embedding on its chunk),
    // with the (mean, M2) of each 64-column part; one warp per (row, part), two columns a lane
    const int lane = W.t & 31;
    const long long gw = gtid >> 5, nw = gthreads >> 5;
    for (int e = 0; e < P.n_experts; ++e) {
      const ExpertRT& X = P.ex[e];
      const long long items = (long long)P.B * X.S * nparts;
      for (long long it = gw; it < items; it += nw) {
        const int part = (int)(it % nparts);
        const long long row = it / nparts;
        const int b = (int)(row / X.S), pos = (int)(row % X.S);
        const int col = part * kStatCols + 2 * lane;
        float v0 = z0_at(P, b, pos, col) + X.pos[(size_t)pos * D + col];
        float v1 = z0_at(P, b, pos, col + 1) + X.pos[(size_t)pos * D + col + 1];
        if (pos >= X.start) { v0 += X.temb[col]; v1 += X.temb[col + 1]; }
        *reinterpret_cast<float2*>(X.x32[0] + (size_t)row * D + col) = make_float2(v0, v1);
        *reinterpret_cast<__half2*>(X.x16[0] + tidx(P.B * X.S, (int)row, col)) = __floats2half2_rn(v0, v1);
        float sum = v0 + v1;
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, off);
        const float mean = sum / (float)kStatCols;
        float m2 = (v0 - mean) * (v0 - mean) + (v1 - mean) * (v1 - mean);
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) m2 += __shfl_xor_sync(0xffffffffu, m2, off);
        if (lane == 0) X.xstat[0][(size_t)row * nparts + part] = make_float2(mean, m2);
      }
    }
    // the context rows, tiled for the cross K/V projection's activation copies
    for (long long i = gtid; i < (long long)P.B * P.C * D; i += gthreads) {
      const int r = (int)(i / D), c = (int)(i % D);
      P.ctx16[tidx(P.B * P.C, r, c)] = P.ctx[i];
    }
    // context LayerNorm statistics (two-pass), one warp per row
    const long long crows = (long long)P.B * P.C;
    for (long long r = gw; r < crows; r += nw) {
      float s = 0.f;
      for (int c = lane; c < D; c += 32) s += __half2float(P.ctx[r * D + c]);
#pragma unroll
      for (int off = 16; off > 0; off >>= 1) s += __shfl_xor_sync(0xffffffffu, s, off);
      const float mean = s / D;
      float q = 0.f;
      for (int c = lane; c < D; c += 32) { const float d = __half2float(P.ctx[r * D + c]) - mean; q += d * d; }
#pragma unroll
      for (int off = 16; off > 0; off >>= 1) q += __shfl_xor_sync(0xffffffffu, q, off);
      if (lane == 0) P.ctxstat[r] = make_float2(mean, rsqrtf(q / D + 1e-5f));
    }
  }
  if (P.mode != CFB_MODE_FLOW) {
    // chain: W beams per request, cum = [0, -inf, ...] (flow_proposer.py:1220-1224)
    // tree: a one-node frontier per request, cum = 0 (flow_proposer.py:1289-1292)
    // lastp is request-major: beam w of request b is row b * Wmax + w
    const bool treem = (P.mode == CFB_MODE_TREE || P.mode == CFB_MODE_BEAM_TREE);
    const int Wm = P.Wmax, per = treem ? 1 : Wm;
    for (long long i = gtid; i < (long long)P.B * per; i += gthreads) {
      const int b = (int)(i / per), w = (int)(i % per);
      for (int j = 0; j < P.order; ++j)
        P.lastp[((size_t)b * Wm + w) * P.order + j] = (j == 0) ? P.known0[b] : -1;
    }
    for (long long i = gtid; i < (long long)P.B * Wm; i += gthreads)
      P.cum[i] = (i % Wm == 0) ? 0.f : -INFINITY;
    // depth-1 head-input side rows, straight from the committed token
    path_gather(P, per, P.B * per, 0, P.B * per, 1, true, gtid, gthreads);
  }
}

// ------------------------------------------------------------------------------------------
// after the head GEMM: every CTA publishes its (max, sumexp, top-TB) per beam row, merging the
// row's slice lanes (their sorted lists) by TB rounds of a lane argmax
__device__ __noinline__ void head_post(const Plan& P, const Phase& ph, const Job* jt, HeadState& H, const Grp& E) {
  const int rows = ph.rows, TB = ph.topb;
  const RowMap M = head_map(rows, E.t, E.n);
  float m = H.m, ssum = H.s;
  lse_lanes(m, ssum, M.sl);
  float* hp = P.hpart + ((size_t)blockIdx.x * kRowsMax + M.r) * kHeadPartFloats;
  const bool writer = M.q == 0 && M.r < rows;
  if (writer) { __stcg(hp + 0, m); __stcg(hp + 1, ssum); }
  int nxt = 0;
#pragma unroll 1
  for (int round = 0; round < TB; ++round) {
    float v; int id;
    list_at(H, nxt, v, id);
    int own = M.q;
    argmax_lanes(v, id, own, M.sl);
    if (own == M.q) ++nxt;
    if (writer) {
      // pass B of the two-pass head: candidate column -> shortlist row
      const int* cand = jt ? jt[0].cand : nullptr;
      const int gid = (cand && id >= 0 && id < jt[0].R) ? __ldcg(cand + id) : id;
      __stcg(hp + 2 + round, v); __stcg(hp + 2 + kTopMax + round, __int_as_float(gid));
    }
  }
}

// Merging published (max, sumexp, sorted top-k) lists. Request b's `fr` frontier rows are each
// given a group of warps. Each thread follows up to kMaxLists of the `nlists` lists of its row
// (list c of row r at src + (c * kRowsMax + r) * kHeadPartFloats). The group combines the
// log-sum-exps in a fixed order and takes the top-TB by TB rounds of a group argmax over the
// list heads (ties: lower shortlist id). Per row it leaves (m, sumexp) in mbuf/sbuf and the
// TB winners in vbuf/ibuf ([row][kTopMax]) in shared memory; the caller synchronises.
constexpr int kMaxLists = 5;
constexpr int kMaxDepth = 8;
struct MergeBufs { float* vbuf; int* ibuf; float* mbuf; float* sbuf; float* wv; int* wid; int* wown; float* wm; float* ws; };
CFB_DEV MergeBufs merge_bufs(Smem& S) {
  MergeBufs M;
  M.vbuf = S.scratch;
  M.ibuf = reinterpret_cast<int*>(M.vbuf + kTopMax * kTopMax);
  M.mbuf = reinterpret_cast<float*>(M.ibuf + kTopMax * kTopMax);
  M.sbuf = M.mbuf + kTopMax;
  M.wv = M.sbuf + kTopMax;
  M.wid = reinterpret_cast<int*>(M.wv + 32);
  M.wown = M.wid + 32;
  M.wm = reinterpret_cast<float*>(M.wown + 32);
  M.ws = M.wm + 32;
  return M;
}
constexpr int kMergeFloats = 2 * kTopMax * kTopMax + 2 * kTopMax + 5 * 32;   // floats merge_bufs uses

CFB_DEV void merge_rows(const Plan& P, const float* src, int nlists, int b, int fr, int TB, const MergeBufs& M,
                        const Grp& W) {
  const int warp = W.t >> 5, lane = W.t & 31, nwarps = W.n >> 5;
  const int wpg = max(1, nwarps / fr);              // warps per frontier row
  const int grp = warp / wpg, gt = (warp - grp * wpg) * 32 + lane, gn = wpg * 32;
  if (grp >= fr) return;
  const int gbar = 3 + grp;                         // named barrier of this row group
  const int row = b * fr + grp;
  float hv[kMaxLists], nv[kMaxLists];
  int hi[kMaxLists], ni[kMaxLists], pos[kMaxLists];
  float m = -INFINITY, ssum = 0.f;
#pragma unroll
  for (int l = 0; l < kMaxLists; ++l) {
    const int c = gt + l * gn;
    hv[l] = nv[l] = -INFINITY; hi[l] = ni[l] = 0x7fffffff; pos[l] = 0;
    if (c < nlists) {
      const float* hp = src + ((size_t)c * kRowsMax + row) * kHeadPartFloats;
      const float mb = __ldcg(hp), sb = __ldcg(hp + 1);
      hv[l] = __ldcg(hp + 2); hi[l] = __float_as_int(__ldcg(hp + 2 + kTopMax));
      if (TB > 1) { nv[l] = __ldcg(hp + 3); ni[l] = __float_as_int(__ldcg(hp + 3 + kTopMax)); }
      lse_merge(m, ssum, mb, sb);
    }
  }
  lse_lanes(m, ssum, 32);
  if (lane == 0) { M.wm[warp] = m; M.ws[warp] = ssum; }
  asm volatile("bar.sync %0, %1;" :: "r"(gbar), "r"(gn) : "memory");
  m = M.wm[grp * wpg]; ssum = M.ws[grp * wpg];
  for (int w = 1; w < wpg; ++w) lse_merge(m, ssum, M.wm[grp * wpg + w], M.ws[grp * wpg + w]);
  if (gt == 0) { M.mbuf[grp] = m; M.sbuf[grp] = ssum; }
#pragma unroll 1
  for (int round = 0; round < TB; ++round) {
    float v = -INFINITY; int id = 0x7fffffff, ol = 0;
#pragma unroll
    for (int l = 0; l < kMaxLists; ++l) if (better(hv[l], hi[l], v, id)) { v = hv[l]; id = hi[l]; ol = l; }
    int own = gt;
    argmax_lanes(v, id, own, 32);
    asm volatile("bar.sync %0, %1;" :: "r"(gbar), "r"(gn) : "memory");   // last round's reads done
    if (lane == 0) { M.wv[warp] = v; M.wid[warp] = id; M.wown[warp] = own; }
    asm volatile("bar.sync %0, %1;" :: "r"(gbar), "r"(gn) : "memory");
    v = M.wv[grp * wpg]; id = M.wid[grp * wpg]; own = M.wown[grp * wpg];
    for (int w = 1; w < wpg; ++w) {
      const float vo = M.wv[grp * wpg + w]; const int io = M.wid[grp * wpg + w], oo = M.wown[grp * wpg + w];
      if (better(vo, io, v, id) || (vo == v && io == id && oo < own)) { v = vo; id = io; own = oo; }
    }
    if (own == gt) {               // the winner moves on in the list it came from
#pragma unroll
      for (int l = 0; l < kMaxLists; ++l) {
        if (l != ol) continue;
        hv[l] = nv[l]; hi[l] = ni[l]; ++pos[l];
        nv[l] = -INFINITY; ni[l] = 0x7fffffff;
        if (pos[l] + 1 < TB) {
          const float* hp = src + ((size_t)(gt + l * gn) * kRowsMax + row) * kHeadPartFloats;
          nv[l] = __ldcg(hp + 3 + pos[l]); ni[l] = __float_as_int(__ldcg(hp + 3 + kTopMax + pos[l]));
        }
      }
    }
    if (gt == 0) { M.vbuf[grp * kTopMax + round] = v; M.ibuf[grp * kTopMax + round] = id; }
  }
}

// Rank-local merge of a row-sharded head (PK_RMERGE): request b's rows of this rank's CTA lists
// merged into one list per row in xloc, for the caller to gather across ranks.
__device__ __noinline__ void rmerge_phase(const Plan& P, const Phase& ph, Smem& S, const Grp& W) {
  const MergeBufs M = merge_bufs(S);
  const int fr = ph.fr, TB = ph.topb;
  for (int b = blockIdx.x; b < P.B; b += P.G) {
    merge_rows(P, P.hpart, P.G, b, fr, TB, M, W);
    gsync(W);
    for (int e = W.t; e < fr * kHeadPartFloats; e += W.n) {
      const int r = e / kHeadPartFloats, f = e - r * kHeadPartFloats;
      float v;
      if (f == 0) v = M.mbuf[r];
      else if (f == 1) v = M.sbuf[r];
      else if (f < 2 + kTopMax) v = (f - 2 < TB) ? M.vbuf[r * kTopMax + f - 2] : -INFINITY;
      else v = __int_as_float((f - 2 - kTopMax < TB) ? M.ibuf[r * kTopMax + f - 2 - kTopMax] : 0x7fffffff);
      __stcg(P.xloc + (size_t)(b * fr + r) * kHeadPartFloats + f, v);
    }
    gsync(W);
  }
}

// The beam phase: one CTA per request (reference flow_proposer.py:1234-1259 chain, :1295-1331
// tree). The frontier rows' lists are merged (the CTAs' lists, or for a row-sharded head the
// ranks' gathered lists), then one thread picks the survivors from shared memory and all
// threads write the new frontier and gather the next depth's path and markov rows.
__device__ __noinline__ void beam_phase(const Plan& P, const Phase& ph, Smem& S, const Grp& W, unsigned long long* prow) {
  const bool treem = (ph.post == PO_BEAM_TREE);
  const int fr = ph.fr, TB = ph.topb, order = P.order, step = ph.step, Wm = P.Wmax;
  const int TB2 = treem ? TB : P.width;
  const int k = treem ? min(ph.keep, fr * TB2) : P.width;
  const MergeBufs M = merge_bufs(S);
  float* lp = M.vbuf;                                             // merged values become log-probs
  int* lid = M.ibuf;
  float* cumo = S.scratch + kMergeFloats;                         // [kTopMax] cum before the step
  float* selc = cumo + kTopMax;                                   // [kTopMax] cum after it
  int* sel = reinterpret_cast<int*>(selc + kTopMax);              // [kTopMax] chosen candidate
  int* hb = sel + kTopMax;                                        // [kMaxDepth][kTopMax] back-pointers
  int64_t* oldp = reinterpret_cast<int64_t*>(hb + kMaxDepth * kTopMax);   // [kTopMax][order]
  int64_t* ht = oldp + kTopMax * 8;                               // [kMaxDepth][kTopMax] tokens
  const bool sharded = P.nranks > 1;
  for (int b = blockIdx.x; b < P.B; b += P.G) {
    if (W.t < fr) cumo[W.t] = P.cum[b * Wm + W.t];
    for (int e = W.t; e < fr * order; e += W.n)
      oldp[e] = P.lastp[((size_t)b * Wm + e / order) * order + e % order];
    merge_rows(P, sharded ? P.xall : P.hpart, sharded ? P.nranks : P.G, b, fr, TB, M, W);
    gsync(W);
    if (prow && W.t == 0) prow[16] = globaltimer();
    // log-probs of the merged top-TB per row
    if (W.t < fr * TB) {
      const int r = W.t / TB, i = W.t - r * TB;
      const float mm = M.mbuf[r], ss = M.sbuf[r];
      const bool okrow = (ss > 0.f) && isfinite(mm) && isfinite(ss);
      const float lse = okrow ? mm + logf(ss) : 0.f;
      const float v = lp[r * kTopMax + i];
      const int id = lid[r * kTopMax + i];
      const bool ok = okrow && id >= 0 && id < P.R && !isnan(v) && v != -INFINITY;
      lp[r * kTopMax + i] = ok ? v - lse : -INFINITY;
      lid[r * kTopMax + i] = ok ? id : 0;
    }
    gsync(W);
    // survivors: the best k of cum[w] + lp[w][i] (one thread, shared memory only)
    if (W.t == 0) {
      HeadState C; head_reset(C);     // tv = cumulative log-prob, ti = w * TB2 + i
#pragma unroll 1
      for (int w = 0; w < fr; ++w)
#pragma unroll 1
        for (int i = 0; i < TB2; ++i) top_insert(C, k, cumo[w] + lp[w * kTopMax + i], w * TB2 + i);
#pragma unroll 1
      for (int i = 0; i < k; ++i) {
        float cv; int cid;
        list_at(C, i, cv, cid);
        // candidate ids are < fr * TB2 by construction; clamp anyway so that no value read back
        // from memory can ever become an out-of-range index
        sel[i] = min(max(cid, 0), fr * TB2 - 1);
        selc[i] = cv;
      }
    }
    gsync(W);
    // the new frontier: path rows, cum, and this depth's tokens
    for (int e = W.t; e < k * order; e += W.n) {
      const int i = e / order, j = e - i * order;
      const int src = sel[i] / TB2, ii = sel[i] - src * TB2;
      int64_t v;
      if (j == 0) {
        const int loc = lid[src * kTopMax + ii];
        v = (loc >= 0 && loc < P.R) ? P.shortlist[loc] : (int64_t)0;
        P.cum[b * Wm + i] = selc[i];
        if (treem) {
          P.tokens[(size_t)b * 2 * P.N + ph.base + i] = v;
          P.tokens[(size_t)b * 2 * P.N + P.N + ph.base + i] = (step == 1) ? (int64_t)-1 : (int64_t)(ph.base_prev + src);
        } else {
          P.toks[((size_t)(step - 1) * P.B + b) * P.width + i] = v;
          P.bps[((size_t)(step - 1) * P.B + b) * P.width + i] = src;
        }
      } else {
        v = oldp[src * order + j - 1];
      }
      P.lastp[((size_t)b * Wm + i) * order + j] = v;
    }
    gsync(W);
    if (prow && W.t == 0) prow[17] = globaltimer();
    if (!treem && ph.last) {
      // walk the best beam back (flow_proposer.py:1261-1267); argmax keeps the first maximum.
      // Every depth's tokens and back-pointers are staged first, in parallel.
      const int Wd = P.width;
      for (int e = W.t; e < step * Wd; e += W.n) {
        ht[e] = P.toks[((size_t)(e / Wd) * P.B + b) * Wd + e % Wd];
        hb[e] = P.bps[((size_t)(e / Wd) * P.B + b) * Wd + e % Wd];
      }
      gsync(W);
      if (W.t == 0) {
        int idx = 0;
        for (int i = 1; i < Wd; ++i) if (selc[i] > selc[idx]) idx = i;
        for (int s2 = step; s2 >= 1; --s2) {
          P.tokens[(size_t)b * P.depth + (s2 - 1)] = ht[(s2 - 1) * Wd + idx];
          idx = min(max(hb[(s2 - 1) * Wd + idx], 0), Wd - 1);
        }
      }
    }
    gsync(W);
    if (prow && W.t == 0) prow[18] = globaltimer();
  }
}

// The next depth's path-GEMM and markov rows of every request (the embedding rows of the live
// path tokens the beam phase just wrote), spread over the whole grid: one request's rows are
// about 100 KB of scattered embedding rows, too slow for the one CTA that ran its beam step.
__device__ __noinline__ void gather_phase(const Plan& P, const Phase& ph, const Grp& W) {
  const long long t = (long long)blockIdx.x * W.n + W.t, nt = (long long)P.G * W.n;
  path_gather(P, ph.fr, P.B * ph.fr, 0, P.B * ph.fr, min(ph.step, P.order), false, t, nt);
}

// ---- the two-pass candidate head (reference CF_TWOPASS_M with a shared candidate set,
// flow_proposer.py:1142-1184) --------------------------------------------------------------
// Pass A input: the marginal hiddens pred[b, 1 + j] (j < tp_n) as fp16 head-input rows, zero in
// the markov columns (pass A has no markov bias).
__device__ __noinline__ void tpxa_phase(const Plan& P, const Grp& W) {
  const int D = P.D, K = D + P.rank, n = P.tp_n, rows = P.B * n;
  const long long nt = (long long)P.G * W.n;
  for (long long i = (long long)blockIdx.x * W.n + W.t; i < (long long)rows * K; i += nt) {
    const int r = (int)(i / K), c = (int)(i - (long long)r * K);
    const int b = r / n, j = r - b * n;
    const float v = c < D ? P.pred[((size_t)b * P.DL + 1 + j) * D + c] : 0.f;
    P.txa[tidx(rows, r, c)] = __float2half_rn(v);
  }
}

// Histogram increment aggregated over the lanes of a warp that hit the same bin (the keys of
// one request crowd into few bins, and same-address shared atomics serialise). All lanes of the
// warp must call it; `live` = false contributes nothing.
CFB_DEV void hist_add(unsigned* hist, unsigned bin, bool live) {
  const unsigned act = __ballot_sync(0xffffffffu, live);
  if (!act) return;
  const int lane = threadIdx.x & 31, first = __ffs(act) - 1;
  const unsigned b0 = __shfl_sync(0xffffffffu, bin, first);
  if (__all_sync(0xffffffffu, !live || bin == b0)) {          // the common case: one bin
    if (lane == first) atomicAdd(&hist[b0], (unsigned)__popc(act));
    return;
  }
  const unsigned same = __match_any_sync(0xffffffffu, live ? bin : 0xffffffffu) & act;
  if (live && lane == __ffs(same) - 1) atomicAdd(&hist[bin], (unsigned)__popc(same));
}

// order-preserving map of a float to uint32 (larger float -> larger key)
CFB_DEV unsigned float_key(float f) {
  const unsigned u = __float_as_uint(f);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

// ---- pass A's top-tp_m selection, over the whole grid: keys, then a byte-wise radix select ----
// Each CTA owns a contiguous range of the B x tp_rs keys (at most two requests, since G >= B).
struct KeyRange { long long e0, e1; int b0, b1; };
CFB_DEV KeyRange key_range(const Plan& P) {
  const long long total = (long long)P.B * P.tp_rs, per = (total + P.G - 1) / P.G;
  KeyRange kr;
  kr.e0 = min(total, (long long)blockIdx.x * per);
  kr.e1 = min(total, kr.e0 + per);
  kr.b0 = (int)(kr.e0 / P.tp_rs);
  kr.b1 = kr.e1 > kr.e0 ? (int)((kr.e1 - 1) / P.tp_rs) : kr.b0 - 1;
  return kr;
}

// The select state after `passes` radix passes of request b (one warp, every lane gets it):
// the key prefix so far, its mask, and how many keys equal to the prefix are still needed.
// cnt(>= bin) is a suffix sum over the lanes' 8 bins each; the digit is the bin where the count
// from the top first reaches `need`.
CFB_DEV void radix_state(const Plan& P, int b, int passes, unsigned& prefix, unsigned& pmask, int& need) {
  const int lane = threadIdx.x & 31;
  prefix = 0u; pmask = 0u; need = P.tp_m;
  for (int p = 0; p < passes; ++p) {
    const int shift = 24 - 8 * p;
    const uint4* hp = reinterpret_cast<const uint4*>(P.thist + ((size_t)p * P.B + b) * 256) + 2 * lane;
    const uint4 h0 = __ldcg(hp), h1 = __ldcg(hp + 1);
    const unsigned h[8] = {h0.x, h0.y, h0.z, h0.w, h1.x, h1.y, h1.z, h1.w};
    int c = 0;
#pragma unroll
    for (int i = 0; i < 8; ++i) c += (int)h[i];
    int suf = c;                                         // keys in bins >= 8 * lane
#pragma unroll
    for (int off = 1; off < 32; off <<= 1) {
      const int o = __shfl_down_sync(0xffffffffu, suf, off);
      if (lane + off < 32) suf += o;
    }
    const unsigned hit = __ballot_sync(0xffffffffu, suf >= need);
    const int L = hit ? 31 - __clz(hit) : 0;             // the highest lane whose suffix reaches need
    const int above = __shfl_sync(0xffffffffu, suf - c, L);   // keys in bins above lane L's
    int d = 0, nd = 0;
    if (lane == L) {
      int cum = above, i = 7;
      for (; i > 0; --i) {
        if (cum + (int)h[i] >= need) break;
        cum += (int)h[i];
      }
      d = 8 * L + i; nd = need - cum;
    }
    d = __shfl_sync(0xffffffffu, d, L);
    nd = __shfl_sync(0xffffffffu, nd, L);
    prefix |= (unsigned)d << shift;
    pmask |= 255u << shift;
    need = nd;
  }
}

// Keys of this CTA's range (and, for pass 0, the histogram of their top byte): the log-sum-exp
// of each marginal row from the head phase's per-CTA (max, sumexp), each shortlist row's best
// log-prob over the depths as an order-preserving uint32 (row stride padded to 4 with zeros).
// pass > 0 (PK_TPRAD): the histogram of byte `pass` of the keys that match the prefix so far.
__device__ __noinline__ void tprad_phase(const Plan& P, Smem& S, const Grp& W, int pass) {
  const KeyRange kr = key_range(P);
  if (kr.e0 >= kr.e1) return;
  const int n = P.tp_n, R = P.R, Rs = P.tp_rs, nb = kr.b1 - kr.b0 + 1;
  const int warp = W.t >> 5, lane = W.t & 31, nw = W.n >> 5;
  unsigned* hist = reinterpret_cast<unsigned*>(S.scratch);                 // [2][256]
  float* lse = reinterpret_cast<float*>(hist + 512);                        // [2][kMaxDepth]
  unsigned* st = reinterpret_cast<unsigned*>(lse + 2 * kMaxDepth);        // [2][2]: prefix, mask
  for (int i = W.t; i < 512; i += W.n) hist[i] = 0u;
  if (pass == 0) {
    for (int q = warp; q < nb * n; q += nw) {
      const int row = (kr.b0 + q / n) * n + q % n;
      float m = -INFINITY, s = 0.f;
      for (int c = lane; c < P.G; c += 32) {
        const float* hp = P.hpart + ((size_t)c * kRowsMax + row) * kHeadPartFloats;
        lse_merge(m, s, __ldcg(hp), __ldcg(hp + 1));
      }
      lse_lanes(m, s, 32);
      if (lane == 0) lse[q] = m + logf(s);
    }
  } else if (warp < nb) {
    unsigned pre, msk; int need;
    radix_state(P, kr.b0 + warp, pass, pre, msk, need);
    if (lane == 0) { st[2 * warp] = pre; st[2 * warp + 1] = msk; }
  }
  gsync(W);
  const int shift = 24 - 8 * pass;
  for (long long e0 = kr.e0 + warp * 32; e0 < kr.e1; e0 += W.n) {   // whole warps
    const long long e = e0 + lane;
    const bool in = e < kr.e1;
    const int b = in ? (int)(e / Rs) : kr.b0, r = in ? (int)(e - (long long)b * Rs) : 0;
    const int bl = b - kr.b0;
    unsigned k = 0u;
    if (pass == 0) {
      if (in && r < R) {
        const float* lg = P.tlog + (size_t)b * n * R + r;
        float v[kMaxDepth];
#pragma unroll
        for (int j = 0; j < kMaxDepth; ++j) v[j] = j < n ? __ldcg(lg + (size_t)j * R) : -INFINITY;
        float best = -INFINITY;
#pragma unroll
        for (int j = 0; j < kMaxDepth; ++j) if (j < n) best = fmaxf(best, v[j] - lse[bl * n + j]);
        k = float_key(best);
      }
      if (in) P.tkeys[e] = k;
    } else if (in) {
      k = __ldcg(P.tkeys + e);
    }
    const bool live = in && r < R && (pass == 0 || (k & st[2 * bl + 1]) == st[2 * bl]);
    hist_add(hist + 256 * bl, (k >> shift) & 255u, live);
  }
  gsync(W);
  for (int i = W.t; i < nb * 256; i += W.n)
    if (hist[i]) atomicAdd(P.thist + ((size_t)pass * P.B + kr.b0 + i / 256) * 256 + (i & 255), hist[i]);
}

// After the four passes: the threshold key T (the tp_m-th largest) and `need` keys equal to it.
// PK_TPCNT: this CTA's counts of keys above and at T, per request. PK_TPSEL: each CTA writes its
// picks at the offset the counts of the CTAs before it give, in ascending shortlist order (ties
// at T go to the lower rows); threads own contiguous sub-ranges placed by one block scan.
__device__ __noinline__ void tpsel_phase(const Plan& P, Smem& S, const Grp& W, bool write) {
  const KeyRange kr = key_range(P);
  if (kr.e0 >= kr.e1) return;
  const int R = P.R, Rs = P.tp_rs, M = P.tp_m, nb = kr.b1 - kr.b0 + 1;
  const int warp = W.t >> 5, lane = W.t & 31, nw = W.n >> 5;
  int* sc = reinterpret_cast<int*>(S.scratch);              // [2][8]: T, need, gbase, ebase; [2 * 32 + 2] scan
  if (warp < nb) {
    const int b = kr.b0 + warp;
    unsigned pre, msk; int need;
    radix_state(P, b, 4, pre, msk, need);
    int gb = 0, eb = 0;
    if (write) {                                            // counts of the CTAs before this one
      for (int c = lane; c < (int)blockIdx.x; c += 32) {
        gb += __ldcg(P.tcnt + ((size_t)b * P.G + c) * 2);
        eb += __ldcg(P.tcnt + ((size_t)b * P.G + c) * 2 + 1);
      }
#pragma unroll
      for (int off = 16; off > 0; off >>= 1) {
        gb += __shfl_xor_sync(0xffffffffu, gb, off);
        eb += __shfl_xor_sync(0xffffffffu, eb, off);
      }
    }
    if (lane == 0) { sc[8 * warp] = (int)pre; sc[8 * warp + 1] = need; sc[8 * warp + 2] = gb; sc[8 * warp + 3] = eb; }
  }
  gsync(W);
  int* scan = sc + 16;
  for (int bl = 0; bl < nb; ++bl) {
    const int b = kr.b0 + bl;
    const long long lo = max(kr.e0, (long long)b * Rs), hi = min(kr.e1, (long long)(b + 1) * Rs);
    const unsigned T = (unsigned)sc[8 * bl];
    const int need = sc[8 * bl + 1];
    const long long chunk = (hi - lo + W.n - 1) / W.n;
    const long long t0 = min(hi, lo + W.t * chunk), t1 = min(hi, t0 + chunk);
    int gt = 0, eq = 0;
    for (long long e = t0; e < t1; ++e) {
      const int r = (int)(e - (long long)b * Rs);
      const unsigned k = __ldcg(P.tkeys + e);
      if (r < R) { gt += k > T; eq += k == T; }
    }
    int ag = gt, ae = eq;
#pragma unroll
    for (int off = 1; off < 32; off <<= 1) {
      const int ug = __shfl_up_sync(0xffffffffu, ag, off), ue = __shfl_up_sync(0xffffffffu, ae, off);
      if (lane >= off) { ag += ug; ae += ue; }
    }
    if (lane == 31) { scan[2 + 2 * warp] = ag; scan[3 + 2 * warp] = ae; }
    gsync(W);
    if (W.t == 0) {
      int sg = 0, se = 0;
      for (int w = 0; w < nw; ++w) {
        const int tg = scan[2 + 2 * w], te = scan[3 + 2 * w];
        scan[2 + 2 * w] = sg; scan[3 + 2 * w] = se;
        sg += tg; se += te;
      }
      scan[0] = sg; scan[1] = se;
    }
    gsync(W);
    if (!write) {
      if (W.t == 0) {
        P.tcnt[((size_t)b * P.G + blockIdx.x) * 2] = scan[0];
        P.tcnt[((size_t)b * P.G + blockIdx.x) * 2 + 1] = scan[1];
      }
    } else {
      const int gbase = sc[8 * bl + 2] + scan[2 + 2 * warp] + ag - gt;
      const int ebase = sc[8 * bl + 3] + scan[3 + 2 * warp] + ae - eq;
      int pos = gbase + min(ebase, need), seen = ebase;
      int* out = P.tcd + (size_t)b * M;
      for (long long e = t0; e < t1; ++e) {
        const int r = (int)(e - (long long)b * Rs);
        if (r >= R) continue;
        const unsigned k = __ldcg(P.tkeys + e);
        // (pos < M always holds: the picks are the rows above T plus `need` rows at T)
        if (k > T) { if (pos < M) out[pos] = r; ++pos; }
        else if (k == T) { if (seen < need && pos < M) out[pos++] = r; ++seen; }
      }
    }
    gsync(W);
  }
}

// The candidate head: the rows tcd of the packed shortlist head, packed in the same layout (cfb_pack.cu)
// as one [B * tp_m, D + rank] matrix, read from the packed full head: a 16 x 16 block of a
// packed matrix holds row g's (and g + 8's) column pairs 2t and 2t + 8 in lane 4g + t. A warp
// takes one 16-row group and a range of 16-column blocks: the two source rows of each lane are
// looked up once, then 4 blocks' loads are in flight at a time.
__device__ __noinline__ void tpgath_phase(const Plan& P, const Grp& W, const uint4* head) {
  // packed layout (cfb_pack_linear): 64-row tiles of [K/64][64 rows][8 swizzled 16-byte chunks]
  const int Kh = (P.D + P.rank + 63) / 64;
  const int nout = P.B * P.tp_m, npad = (nout + 63) / 64 * 64;
  const size_t tile16 = (size_t)Kh * 512;                 // 16-byte words per 64-row tile
  const long long tasks = (long long)npad * Kh * 8;
  const long long gtid = (long long)blockIdx.x * W.n + W.t, gthreads = (long long)P.G * W.n;
  for (long long i = gtid; i < tasks; i += gthreads) {
    const int c = (int)(i & 7);
    const long long rest = i >> 3;
    const int h = (int)(rest % Kh), d = (int)(rest / Kh);
    uint4 v = make_uint4(0u, 0u, 0u, 0u);                  // padding rows of the last tile: zeros
    if (d < nout) {
      int s = __ldcg(P.tcd + d);
      s = min(max(s, 0), P.R - 1);                         // (always in range; never read outside)
      v = __ldg(head + (size_t)(s >> 6) * tile16 + (size_t)h * 512 + (size_t)(s & 63) * 8 + (c ^ (s & 7)));
    }
    P.tchead[(size_t)(d >> 6) * tile16 + (size_t)h * 512 + (size_t)(d & 63) * 8 + (c ^ (d & 7))] = v;
  }
}

// ------------------------------------------------------------------------------------------
// Runs phases [p0, p1) of the plan: the whole table, or one segment of a sharded-head plan.
// The phases that run once per draft or per depth (prep, attention, beam, gathers) are out of
// line, so the GEMM path stays compact in the instruction cache.
template <int MAXNT>
__global__ void __launch_bounds__(kThreads, 1) engine_kernel(const Plan* __restrict__ Pp, int p0, int p1) {
  // The plan record stays in global memory: passed by value (a __grid_constant__ parameter) it
  // measured slower on the head phase (75 vs 68 us a depth at the 4B shape). Each CTA keeps a
  // copy in shared memory instead: a grid barrier's acquire leaves the L1 cold, and every role
  // reads plan fields right after one.
  __shared__ __align__(16) Plan s_plan;
  static_assert(sizeof(Plan) % 8 == 0 && sizeof(Plan) <= 2048, "plan copy");
  for (int i = threadIdx.x; i < (int)(sizeof(Plan) / 8); i += blockDim.x)
    reinterpret_cast<uint64_t*>(&s_plan)[i] = __ldcg(reinterpret_cast<const unsigned long long*>(Pp) + i);
  __syncthreads();
  const Plan& P = s_plan;
  // The narrow classes (jobs of <= 16 rows) measured faster with the per-phase profiling
  // switched at run time (CFB_RUN_PROFILE); the wider ones with the profiling compiled out
  // (their plans record no stamps), which frees registers. Results are the same.
  constexpr bool kLean = MAXNT > 2;
  constexpr bool kProf = !kLean;                  // profiling code present in this instantiation
  using WaitClock = typename std::conditional<kProf, ProfClock, NoClock>::type;
  extern __shared__ __align__(1024) uint8_t smem_dyn[];
  // the tensor cores' 128-byte-swizzled operands need 1024-byte-aligned stages (the host leaves
  // 1024 bytes of slack for this)
  uint8_t* const smem_raw = smem_dyn + ((1024u - (smem_u32(smem_dyn) & 1023u)) & 1023u);
  const SmemLayout L = P.sm;
  Smem S;
  S.ring = smem_raw; S.nstages = L.nstages; S.stage_bytes = L.stage_bytes; S.rp = L.rows_pad; S.nbuf = L.nbuf;
  S.xhalf = L.xhalf;
  S.full = reinterpret_cast<uint64_t*>(smem_raw + L.off_bar);
  S.empty = S.full + L.nstages;
  S.accf = S.empty + L.nstages;
  S.acce = S.accf + 2;
  S.fin = S.acce + 2;
  S.slots = reinterpret_cast<float*>(smem_raw + L.off_slots);
  S.scratch = reinterpret_cast<float*>(smem_raw + L.off_scratch);
  S.red = reinterpret_cast<float*>(smem_raw + L.off_red);
  S.rowstat = reinterpret_cast<float2*>(smem_raw + L.off_rowstat);
  S.tbias = reinterpret_cast<float*>(smem_raw + L.off_tile);
  S.tcsum = S.tbias + kTileRows;
  S.flag = reinterpret_cast<int*>(smem_raw + L.off_misc);
  S.phase_ready = reinterpret_cast<volatile int*>(smem_raw + L.off_misc + 4);
  S.desc_ready = reinterpret_cast<volatile int*>(smem_raw + L.off_misc + 8);
  S.desc = smem_raw + L.off_desc;
  const int tid = threadIdx.x, warp = tid >> 5;
  __shared__ uint32_t s_tmem;
  // two accumulators (nbuf) of kAccCols columns
  constexpr uint32_t tmem_cols = 2u * kAccCols;
  static_assert(tmem_cols == 128u, "a power of two of at least 32 TMEM columns");
  if (warp == 0) tmem_alloc(&s_tmem, tmem_cols);   // the accumulators (one CTA per SM: never contended)
  if (tid == 0) {
    // full: the weight producer's expect_tx arrive + the activation producer's arrive; empty,
    // accf, fin: the MMA warp's tcgen05.commit; acce: the epilogue
    for (int i = 0; i < L.nstages; ++i) { mbar_init(&S.full[i], 2); mbar_init(&S.empty[i], 1); }
    for (int i = 0; i < 2; ++i) { mbar_init(&S.accf[i], 1); mbar_init(&S.acce[i], 1); }
    mbar_init(S.fin, 1);
    *S.phase_ready = -1;
    *S.desc_ready = -1;
    // a plan whose earlier run failed stays failed: this run leaves every output untouched
    *S.flag = ld_volatile_int(P.err) != 0;
    fence_mbar_init();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  S.tmem = s_tmem;
  const bool dead = *S.flag != 0;
  __syncthreads();
  if (warp == kWProdWarp) {
    if ((tid & 31) == 0 && !dead) weight_producer(P, S, p0, p1);
    return;
  }
  if (warp == kXProdWarp) {
    if ((tid & 31) == 0 && !dead) x_producer(P, S, p0, p1);
    return;
  }
  const bool is_epi = warp >= kEpiWarp0;
  const Grp Wk{is_epi ? kMma + (tid - kEpiWarp0 * 32) : tid, kWorkers, kBarWorkers};
  const Grp E{tid - kEpiWarp0 * 32, kEpi, kBarEpi};
  // the wide epilogue group: epilogue threads first (0..127), then worker warps 1..7
  const Grp EW{is_epi ? tid - kEpiWarp0 * 32 : kEpi + tid - 32, kEpiWide, kBarWide};
  uint32_t ci = 0, tseq = 0;
  unsigned epoch = 0;
  bool ok = !dead;
  const bool rec = kProf && P.prof && ((!is_epi && tid == 0) || (is_epi && E.t == 0));
  HeadState H;                   // the head phases' per-row (max, sumexp, top-k) of this thread
  head_reset(H);
  if (ok) {                      // the first phase's descriptors
    __shared__ int s_first;
    if (Wk.t == 0) s_first = desc_wait1(P, S.desc_ready, p0);
    gsync(Wk);
    ok = s_first != 0;
  }
  for (int p = p0; p < p1 && ok; ++p) {
    const Phase& ph = S.dphase(p);
    const Job* jt = ph.kind == PK_GEMM ? phase_jobs(P, S, ph, p) : nullptr;
    unsigned long long* prow = kProf && P.prof ? P.prof + ((size_t)p * P.G + blockIdx.x) * kProfSlots : nullptr;
    unsigned long long* stamp = (kProf && P.prof && Wk.t == 0) ? prow : nullptr;
    WaitClock wc;
    if constexpr (kProf) {
      wc.on = rec;
      wc.full = wc.slot = wc.first = wc.last = 0;
      wc.part = wc.atom = wc.fix = wc.tdone = wc.rstat = 0;
    }
    if (stamp) stamp[0] = globaltimer();
    if (Wk.t == 0) *S.phase_ready = p;
    if (ph.kind == PK_PREP) {
      prep_phase(P, Wk);
    } else if (ph.kind == PK_ATTN) {
      attn_phase(P, ph, phase_tasks(P, S, ph, p), S, Wk);
    } else if (ph.kind == PK_BEAM) {
      beam_phase(P, ph, S, Wk, P.prof ? prow : nullptr);
    } else if (ph.kind == PK_GATHER) {
      gather_phase(P, ph, Wk);
    } else if (ph.kind == PK_TPXA) {
      tpxa_phase(P, Wk);
    } else if (ph.kind == PK_TPKEY) {
      tprad_phase(P, S, Wk, 0);
    } else if (ph.kind == PK_TPRAD) {
      tprad_phase(P, S, Wk, ph.step);
    } else if (ph.kind == PK_TPCNT) {
      tpsel_phase(P, S, Wk, false);
    } else if (ph.kind == PK_TPSEL) {
      tpsel_phase(P, S, Wk, true);
    } else if (ph.kind == PK_TPGATH) {
      tpgath_phase(P, Wk, P.tp_head);
    } else if (ph.kind == PK_RMERGE) {
      rmerge_phase(P, ph, S, Wk);
    } else {
      // wide-row builds widen the epilogue of GEMM phases onto worker warps 1..7
      const bool wide = kLean;
      if (is_epi) {
        if (ph.post != PO_NONE) head_reset(H);
        epi_phase(P, ph, jt, tseq, S, H, wide ? EW : E, true, wc);
        if (ph.post != PO_NONE) head_post(P, ph, jt, H, wide ? EW : E);
        if (rec) {
          prow[5] = wc.slot; prow[6] = globaltimer();
          prow[12] = wc.part; prow[13] = wc.atom; prow[14] = wc.fix; prow[15] = wc.tdone;
          prow[19] = wc.rstat;
        }
      } else {
        if (warp == kMmaIssueWarp) {
          tc_phase<WaitClock>(P, ph, jt, ci, tseq, S, wc);
        } else if (wide) {
          if (ph.post != PO_NONE) head_reset(H);
          epi_phase(P, ph, jt, tseq, S, H, EW, false, wc);
          if (ph.post != PO_NONE) head_post(P, ph, jt, H, EW);
        }
        if (rec) { prow[3] = wc.full; prow[4] = wc.slot; prow[10] = wc.first; prow[11] = wc.last; }
      }
    }
    if (stamp) stamp[1] = globaltimer();
    ok = grid_sync(P, epoch, Wk, S.desc_ready, p + 1 < p1 ? p + 1 : -1);
    if (stamp) stamp[2] = globaltimer();
  }
  if (Wk.t == 0) {
    *S.phase_ready = 1 << 30;     // release the activation producer if the loop ended early
    __threadfence();
    const unsigned old = atomicAdd(P.exitcnt, 1u);
    if (old + 1 == (unsigned)P.G) { *P.bar = 0u; *P.exitcnt = 0u; __threadfence(); }
  }
  // every MMA this CTA issued has completed (the epilogue's TMEM reads are behind the last grid
  // barrier) before its tensor memory is freed
  static_assert(kMmaIssueWarp == 0, "the MMA warp also allocates and frees the tensor memory");
  if (warp == 0) {
    tc_commit_warp(S.fin);
    if (tid == 0) mbar_wait(S.fin, 0);
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(S.tmem, tmem_cols);
  }
}

}  // namespace cfb

// ============================================================================================
// host side: lowering a (drafter, run) pair to the phase table
// ============================================================================================
namespace {

thread_local char g_cuda_err[256] = "";

cfb_status cuda_fail(cudaError_t e, const char* what) {
  snprintf(g_cuda_err, sizeof(g_cuda_err), "%s: %s", what, cudaGetErrorString(e));
  return CFB_ERR_CUDA;
}

}  // namespace

cfb_status cfb_launch_status(const char* what) {
  const cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? CFB_OK : cuda_fail(e, what);
}

namespace {

struct Arena {
  size_t off = 0;
  size_t take(size_t bytes, size_t align = 256) {
    off = (off + align - 1) / align * align;
    const size_t o = off;
    off += bytes;
    return o;
  }
};

// fixed offsets at the start of every workspace: plan record, then the 64-byte barrier block
// (bar, exitcnt, spare, err; launch record at +32)
constexpr size_t kOffPlan = 0;
size_t off_barrier() { Arena A; A.take(sizeof(cfb::Plan)); return A.take(64); }

struct Builder {
  const cfb_drafter* d;
  const cfb_run* r;
  uint8_t* base;                 // device base (pointer arithmetic only)
  Arena A;
  std::vector<cfb::Phase> phases;
  std::vector<cfb::Job> jobs;
  std::vector<cfb::AttnTask> attn;
  std::vector<int> segs;         // first phase of every launch segment after the first
  cfb::Plan P{};
  size_t off_phases = 0, off_jobs = 0, off_attn = 0;
  int max_tiles = 0;
  bool too_big = false;          // a phase's units x grid overflows the kernel's 32-bit range math
  int G = 148;                   // persistent grid the phases are cut for
  // a VAE side plan (cfb_vae_plan_build): d / r are stand-ins carrying D, batch and rows
  const cfb_vae_side* vae = nullptr;
  int vrows = 0, vdecode = 0;
  const void* vin = nullptr; void* vout = nullptr;
  template <class T> T* dptr(size_t off) { return reinterpret_cast<T*>(base + off); }
};

bool lin_ok(const cfb_linear& l, int nout, int k) {
  return l.w && l.nout == nout && l.k == k && (k % 16) == 0 &&
         (reinterpret_cast<uintptr_t>(l.w) % 16) == 0;
}

cfb::Job make_job(const cfb_linear& L, int rows) {
  cfb::Job J{};
  J.w = static_cast<const uint4*>(L.w);
  J.Mt = (L.nout + cfb::kTileRows - 1) / cfb::kTileRows;
  J.Kt = L.k / 16;
  J.Kstride = (L.k + 63) / 64 * 4;       // the packed tile's k extent (whole 64-k halves), in 16-k blocks
  J.nkc = (J.Kt + cfb::kUnitK - 1) / cfb::kUnitK;
  J.rows = rows;
  J.nout = L.nout;
  J.xR = rows; J.xcopy = rows; J.oR = rows;
  J.gin = rows > 0 ? rows : 1; J.gstride = 0; J.goff = 0;
  J.bias = L.bias;
  J.colsum = L.colsum;
  return J;
}

void add_phase(Builder& B, cfb::Phase ph, const std::vector<cfb::Job>& js) {
  ph.kind = cfb::PK_GEMM;
  ph.job0 = (int)B.jobs.size();
  ph.njobs = (int)js.size();
  long long u = 0; int t = 0;
  for (auto j : js) {
    j.unit_base = (int)u; j.tile_base = t;
    u += (long long)j.Mt * j.nkc; t += j.Mt;
    B.jobs.push_back(j);
  }
  ph.nunits = (int)u; ph.ntiles = t;
  if ((unsigned long long)u * (unsigned long long)(B.G + 1) >= (1ull << 32)) B.too_big = true;
  // Whole tiles per CTA (no cross-CTA fixup) unless splitting tiles finishes sooner even after
  // paying for the fixup, which costs about as much as streaming kFixupUnits units.
  long long nkc_max = 1;
  int rows_max = 1;
  for (const auto& j : js) { nkc_max = std::max<long long>(nkc_max, j.nkc); rows_max = std::max(rows_max, j.rows); }
  const long long kFixupUnits = rows_max > 16 ? CFB_FIXUP_UNITS_WIDE : CFB_FIXUP_UNITS;
  const long long G = B.G;
  const long long whole_units = (t + G - 1) / G * nkc_max;
  const long long split_units = (u + G - 1) / G + kFixupUnits;
  ph.whole = whole_units <= split_units ? 1 : 0;
  B.max_tiles = std::max(B.max_tiles, t);
  B.phases.push_back(ph);
}

cfb_status lower(Builder& B, size_t* bytes) {
  const cfb_drafter& d = *B.d;
  const cfb_run& r = *B.r;
  const int D = d.hidden, Bq = r.batch, C = d.ctx_rows, DL = d.draft_len, E = d.n_experts;
  const int mode = r.mode;
  const bool vae = B.vae != nullptr;
  if (vae ? mode != cfb::kModeVae : (mode < CFB_MODE_FLOW || mode > CFB_MODE_BEAM_TREE)) return CFB_ERR_INVALID_ARG;
  const bool flow = !vae && (mode == CFB_MODE_FLOW || mode == CFB_MODE_CHAIN || mode == CFB_MODE_TREE);
  const bool beam = !vae && mode != CFB_MODE_FLOW;
  const bool tree = !vae && (mode == CFB_MODE_TREE || mode == CFB_MODE_BEAM_TREE);
  if (vae) {
    const cfb_vae_side& v = *B.vae;
    const int S = B.vrows, FF = v.layers > 0 ? v.layer[0].ffn_up.nout : 64;
    if (!B.vin || !B.vout || !v.pos || (v.layers > 0 && !v.layer)) return CFB_ERR_INVALID_ARG;
    if (v.in_dim <= 0 || v.in_dim % 16 || v.width != D || v.out_dim <= 0 || v.out_dim % 16 || v.layers < 0 ||
        v.heads <= 0 || D % v.heads || (D / v.heads) % 4 || S <= 0 || S > v.max_len || Bq * S > cfb::kRowsMax ||
        FF % cfb::kStatCols)
      return CFB_ERR_UNSUPPORTED;
    if (3 * S * (D / v.heads) + S * S > (cfb::kSmemBudget / 4) / 2) return CFB_ERR_UNSUPPORTED;
    if (!lin_ok(v.in_proj, D, v.in_dim) || !v.in_proj.bias || !lin_ok(v.out_proj, v.out_dim, D) ||
        !v.out_proj.bias || !v.out_proj.colsum)
      return CFB_ERR_INVALID_ARG;
    for (int l = 0; l < v.layers; ++l) {
      const cfb_vae_layer& ly = v.layer[l];
      if (!lin_ok(ly.qkv, 3 * D, D) || !ly.qkv.colsum || !lin_ok(ly.attn_out, D, D) || !lin_ok(ly.ffn_up, FF, D) ||
          !ly.ffn_up.colsum || !lin_ok(ly.ffn_down, D, FF))
        return CFB_ERR_INVALID_ARG;
    }
  }
  if (D <= 0 || D % cfb::kStatCols || Bq <= 0) return CFB_ERR_UNSUPPORTED;
  if (E <= 0 || E > cfb::kMaxExperts || d.chunk <= 0 || E * d.chunk != DL) return CFB_ERR_UNSUPPORTED;
  if (!r.pred) return CFB_ERR_INVALID_ARG;
  if (flow) {
    if (!r.ctx || !d.experts || d.heads <= 0 || D % d.heads || d.layers <= 0 || d.steps <= 0)
      return CFB_ERR_INVALID_ARG;
    if (r.init_mode < CFB_INIT_GIVEN || r.init_mode > CFB_INIT_DELTA || (r.init_mode == CFB_INIT_GIVEN && !r.z0))
      return CFB_ERR_INVALID_ARG;
    if (Bq * DL > cfb::kRowsMax || Bq * C > cfb::kRowsMax) return CFB_ERR_UNSUPPORTED;
    const int hd = D / d.heads, Kmax = std::max(DL, C);
    if (hd % 4 || (DL + 2 * Kmax) * hd + DL * Kmax > (cfb::kSmemBudget / 4) / 2) return CFB_ERR_UNSUPPORTED;
  }
  int Wmax = 0, K = 0;
  if (beam) {
    if (!r.known0 || !r.tokens || !d.shortlist || !d.embed || !d.markov_w1) return CFB_ERR_INVALID_ARG;
    if (d.path_order < 1 || d.path_order > 8 || d.markov_rank <= 0 || d.markov_rank % 16) return CFB_ERR_UNSUPPORTED;
    if (tree) {
      if (r.tree_keep < 1 || r.tree_topb < 1 || r.tree_topb > cfb::kTopMax || r.tree_keep > cfb::kTopMax)
        return CFB_ERR_UNSUPPORTED;
      Wmax = r.tree_keep;
    } else {
      if (r.width < 1 || r.width > cfb::kTopMax) return CFB_ERR_UNSUPPORTED;
      Wmax = r.width;
    }
    K = std::min(r.depth, DL - 1);
    if (K < 1 || (!tree && K != r.depth)) return CFB_ERR_UNSUPPORTED;
    if (Bq * Wmax > cfb::kRowsMax) return CFB_ERR_UNSUPPORTED;
    // the head: every shortlist row, or (row-sharded across ranks) rows [head_row0, +nout)
    if (d.head_row0 < 0 || d.head.nout < 1 || d.head_row0 + d.head.nout > d.shortlist_rows ||
        !lin_ok(d.head, d.head.nout, D + d.markov_rank))
      return CFB_ERR_INVALID_ARG;
    if (r.ranks > 1) {
      if (r.rank < 0 || r.rank >= r.ranks || !r.xloc || !r.xall) return CFB_ERR_INVALID_ARG;
      if (r.ranks > cfb::kMaxLists * 32) return CFB_ERR_UNSUPPORTED;
    } else if (d.head_row0 != 0 || d.head.nout != d.shortlist_rows) {
      return CFB_ERR_INVALID_ARG;     // one GPU holds the whole head
    }
    if (!lin_ok(d.path_offsets, D, d.path_order * D) || !lin_ok(d.path_up, d.path_up.nout, D) ||
        !lin_ok(d.path_down, D, d.path_up.nout) || !d.path_offset_bias || !d.path_down.bias ||
        d.path_up.nout % 16)
      return CFB_ERR_INVALID_ARG;
    // the two-pass head: candidates from the whole head, on one GPU; every request's marginal
    // rows fit one head job
    if (r.twopass_m < 0) return CFB_ERR_INVALID_ARG;
    if (r.twopass_m > 0 && (r.ranks > 1 || r.twopass_m >= d.shortlist_rows || Bq * K > cfb::kRowsMax ||
                            (long long)Bq * r.twopass_m > (1LL << 30)))
      return CFB_ERR_UNSUPPORTED;
  } else if (r.twopass_m != 0) {
    return CFB_ERR_INVALID_ARG;
  }
  const int TPM = beam ? r.twopass_m : 0;
  int G = r.grid;
  if (G <= 0) {
    int dev = 0, sms = 0;
    if (cudaGetDevice(&dev) != cudaSuccess ||
        cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || sms <= 0)
      sms = 148;
    G = sms;
  }
  B.G = G;
  if (TPM && G < Bq) return CFB_ERR_UNSUPPORTED;          // a CTA's key range spans <= 2 requests
  // the beam merge: each thread follows at most kMaxLists of the G published lists per row
  if (beam && (G + 32 * std::max(1, (cfb::kWorkers / 32) / Wmax) - 1) / (32 * std::max(1, (cfb::kWorkers / 32) / Wmax)) > cfb::kMaxLists)
    return CFB_ERR_UNSUPPORTED;
  if (beam && K > cfb::kMaxDepth) return CFB_ERR_UNSUPPORTED;

  Arena& A = B.A;
  A.off = 0;
  A.take(sizeof(cfb::Plan));
  const size_t o_bar = A.take(64);
  const int nparts = D / cfb::kStatCols;
  auto k128 = [](int k) { return (size_t)((k + 127) / 128 * 128); };   // tiled buffers pad K
  std::vector<size_t> o_x32(2 * E), o_x16(2 * E), o_xs(2 * E), o_qkv(E), o_o(E), o_qc(E), o_u(E), o_kvc(E);
  size_t o_ctx16 = 0;
  int FM = 0;
  if (flow) {
    FM = d.experts[0].blocks[0].ffn_up.nout / D;
    if (FM <= 0) return CFB_ERR_INVALID_ARG;
    for (int e = 0; e < E; ++e) {
      const int rows = Bq * (e + 1) * d.chunk;
      for (int q = 0; q < 2; ++q) {
        o_x32[2 * e + q] = A.take((size_t)rows * D * 4);
        o_x16[2 * e + q] = A.take((size_t)rows * k128(D) * 2);
        o_xs[2 * e + q] = A.take((size_t)rows * nparts * 8);
      }
      o_qkv[e] = A.take((size_t)rows * 3 * D * 4);
      o_o[e] = A.take((size_t)rows * k128(D) * 2);
      o_qc[e] = A.take((size_t)rows * D * 4);
      o_u[e] = A.take((size_t)rows * k128(FM * D) * 2);
      o_kvc[e] = A.take((size_t)d.layers * Bq * C * 2 * D * 4);
    }
    o_ctx16 = A.take((size_t)Bq * C * k128(D) * 2);
  }
  const size_t o_ctxs = A.take((size_t)Bq * C * 8);
  size_t o_vin16 = 0, o_vx32 = 0, o_vx16 = 0, o_vxs = 0, o_vqkv = 0, o_vo = 0, o_vu = 0;
  if (vae) {
    const size_t M = (size_t)Bq * B.vrows;
    const int FF = B.vae->layers > 0 ? B.vae->layer[0].ffn_up.nout : 64;
    o_vin16 = A.take(M * k128(B.vae->in_dim) * 2);
    o_vx32 = A.take(M * D * 4);
    o_vx16 = A.take(M * k128(D) * 2);
    o_vxs = A.take(M * nparts * 8);
    o_vqkv = A.take(M * 3 * D * 4);
    o_vo = A.take(M * k128(D) * 2);
    o_vu = A.take(M * k128(FF) * 2);
  }
  const int rank = d.markov_rank, order = d.path_order;
  const int P2 = beam ? d.path_up.nout : 0;
  const int rowsB = Bq * std::max(Wmax, 1);
  size_t o_lastp = 0, o_cum = 0, o_toks = 0, o_bps = 0, o_h16 = 0, o_hstat = 0, o_mpath = 0, o_xhead = 0, o_pg = 0;
  if (beam) {
    o_lastp = A.take((size_t)rowsB * order * 8);
    o_cum = A.take((size_t)rowsB * 4);
    o_toks = A.take((size_t)(K + 1) * rowsB * 8);
    o_bps = A.take((size_t)(K + 1) * rowsB * 4);
    o_h16 = A.take((size_t)rowsB * k128(D) * 2);
    o_hstat = A.take((size_t)rowsB * nparts * 8);
    o_mpath = A.take((size_t)rowsB * k128(P2) * 2);
    o_xhead = A.take((size_t)rowsB * k128(D + rank) * 2);
    o_pg = A.take((size_t)rowsB * k128(order * D) * 2);
  }
  size_t o_txa = 0, o_tlog = 0, o_tkeys = 0, o_tcd = 0, o_tchead = 0, o_thist = 0, o_tcnt = 0;
  if (TPM) {
    const size_t rowsA = (size_t)Bq * K, nc = (size_t)Bq * TPM;
    o_txa = A.take(rowsA * k128(D + rank) * 2);
    o_tlog = A.take(rowsA * d.shortlist_rows * 4);
    o_tkeys = A.take((size_t)Bq * ((d.shortlist_rows + 3) / 4 * 4) * 4);
    o_tcd = A.take(nc * 4);
    o_thist = A.take((size_t)4 * Bq * 256 * 4);
    o_tcnt = A.take((size_t)Bq * G * 2 * 4);
    o_tchead = A.take(cfb_packed_bytes(nc, D + rank));
  }
  const size_t o_gpart = A.take((size_t)G * cfb::kTileRows * cfb::kRowsMax * 4);
  const bool profile = (r.flags & CFB_RUN_PROFILE) != 0;
  const size_t o_hpart = A.take((size_t)G * cfb::kRowsMax * cfb::kHeadPartFloats * 4);

  auto& ph = B.phases; ph.clear();
  B.jobs.clear();
  B.segs.clear();
  auto& at = B.attn; at.clear();
  B.max_tiles = 0;
  B.too_big = false;

  { cfb::Phase p{}; p.kind = cfb::PK_PREP; ph.push_back(p); }

  if (vae) {   // TransformerHiddenVAE encode_sequence / decode_sequence (transformer_hidden.py:51-67)
    const cfb_vae_side& v = *B.vae;
    const int S = B.vrows, M = Bq * S, hd = D / v.heads;
    const int FF = v.layers > 0 ? v.layer[0].ffn_up.nout : 64;
    auto resid_job = [&](const cfb_linear& lin, size_t o_in, int ldin) {
      cfb::Job J = make_job(lin, M);
      J.xkind = cfb::XK_F16; J.x = B.dptr<__half>(o_in); J.ldx = ldin;
      J.ekind = cfb::EK_RESID; J.out32 = B.dptr<float>(o_vx32); J.out16 = B.dptr<__half>(o_vx16); J.ldo = D;
      J.ostats = B.dptr<float2>(o_vxs); J.onparts = nparts;
      return J;
    };
    auto ln_job = [&](const cfb_linear& lin) {
      cfb::Job J = make_job(lin, M);
      J.xkind = cfb::XK_F16; J.x = B.dptr<__half>(o_vx16); J.ldx = D;
      J.ln = cfb::LN_PARTS; J.stats = B.dptr<float2>(o_vxs); J.nparts = nparts;
      return J;
    };
    add_phase(B, cfb::Phase{}, {resid_job(v.in_proj, o_vin16, v.in_dim)});   // x = pos + in_proj(h)
    cfb::AttnTask a{};
    a.q = B.dptr<float>(o_vqkv); a.ldq = 3 * D; a.qoff = 0;
    a.k = a.q; a.ldk = 3 * D; a.koff = D;
    a.v = a.q; a.ldv = 3 * D; a.voff = 2 * D;
    a.out = B.dptr<__half>(o_vo);
    a.rows_per_req = S; a.keys_per_req = S; a.B = Bq; a.hd = hd; a.heads = v.heads;
    a.causal = 0; a.scale = 1.0f / std::sqrt((float)hd); a.outR = M;
    at.push_back(a);
    for (int l = 0; l < v.layers; ++l) {       // pre-LN encoder layers (norm_first, GELU)
      const cfb_vae_layer& ly = v.layer[l];
      cfb::Job J = ln_job(ly.qkv);
      J.ekind = cfb::EK_STORE; J.out32 = B.dptr<float>(o_vqkv); J.ldo = 3 * D;
      add_phase(B, cfb::Phase{}, {J});
      cfb::Phase pa{};
      pa.kind = cfb::PK_ATTN; pa.job0 = 0; pa.njobs = 1; pa.ntiles = Bq * v.heads;
      ph.push_back(pa);
      add_phase(B, cfb::Phase{}, {resid_job(ly.attn_out, o_vo, D)});
      J = ln_job(ly.ffn_up);
      J.ekind = cfb::EK_GELU16; J.out16 = B.dptr<__half>(o_vu); J.ldo = FF;
      add_phase(B, cfb::Phase{}, {J});
      add_phase(B, cfb::Phase{}, {resid_job(ly.ffn_down, o_vu, FF)});
    }
    cfb::Job J = ln_job(v.out_proj);          // final LayerNorm folded in; mu or decoder_out
    J.ldo = v.out_dim;
    if (B.vdecode) { J.ekind = cfb::EK_STORE; J.out32 = static_cast<float*>(B.vout); }
    else { J.ekind = cfb::EK_STORE16; J.out16 = static_cast<__half*>(B.vout); }
    add_phase(B, cfb::Phase{}, {J});
  }

  if (flow) {
    const int L = d.layers, T = d.steps, hd = D / d.heads;
    {   // cross K/V of every (expert, block), once per draft
      std::vector<cfb::Job> js;
      for (int e = 0; e < E; ++e)
        for (int l = 0; l < L; ++l) {
          const cfb_linear& lin = d.experts[e].blocks[l].cross_kv;
          if (!lin_ok(lin, 2 * D, D)) return CFB_ERR_INVALID_ARG;
          cfb::Job J = make_job(lin, Bq * C);
          J.xkind = cfb::XK_F16; J.x = B.dptr<__half>(o_ctx16); J.ldx = D;
          J.ln = cfb::LN_DIRECT; J.stats = B.dptr<float2>(o_ctxs);
          J.ekind = cfb::EK_STORE;
          J.out32 = B.dptr<float>(o_kvc[e]) + (size_t)l * Bq * C * 2 * D; J.ldo = 2 * D;
          js.push_back(J);
        }
      add_phase(B, cfb::Phase{}, js);
    }
    // attention tasks: the E self-attentions first, then the cross-attentions by (block, expert),
    // so that each attention phase covers one contiguous range of tasks
    for (int e = 0; e < E; ++e) {
      const int S = (e + 1) * d.chunk;
      cfb::AttnTask a{};
      a.q = B.dptr<float>(o_qkv[e]); a.ldq = 3 * D; a.qoff = 0;
      a.k = a.q; a.ldk = 3 * D; a.koff = D;
      a.v = a.q; a.ldv = 3 * D; a.voff = 2 * D;
      a.out = B.dptr<__half>(o_o[e]);
      a.rows_per_req = S; a.keys_per_req = S; a.B = Bq; a.hd = hd; a.heads = d.heads;
      a.causal = 1; a.scale = 1.0f / std::sqrt((float)hd); a.outR = Bq * S;
      at.push_back(a);
    }
    for (int l = 0; l < L; ++l)
      for (int e = 0; e < E; ++e) {
        const int S = (e + 1) * d.chunk;
        cfb::AttnTask c{};
        c.q = B.dptr<float>(o_qc[e]); c.ldq = D; c.qoff = 0;
        c.k = B.dptr<float>(o_kvc[e]) + (size_t)l * Bq * C * 2 * D; c.ldk = 2 * D; c.koff = 0;
        c.v = c.k; c.ldv = 2 * D; c.voff = D;
        c.out = B.dptr<__half>(o_o[e]);
        c.rows_per_req = S; c.keys_per_req = C; c.B = Bq; c.hd = hd; c.heads = d.heads;
        c.causal = 0; c.scale = 1.0f / std::sqrt((float)hd); c.outR = Bq * S;
        at.push_back(c);
      }
    auto add_attn = [&](int first) {
      cfb::Phase p{};
      p.kind = cfb::PK_ATTN; p.job0 = first; p.njobs = E; p.ntiles = E * Bq * d.heads;
      ph.push_back(p);
    };
    for (int s = 0; s < T; ++s) {
      const int pb = s & 1;
      auto ln_job = [&](const cfb_linear& lin, int e) {
        const int S = (e + 1) * d.chunk;
        cfb::Job J = make_job(lin, Bq * S);
        J.xkind = cfb::XK_F16; J.x = B.dptr<__half>(o_x16[2 * e + pb]); J.ldx = D;
        J.ln = cfb::LN_PARTS; J.stats = B.dptr<float2>(o_xs[2 * e + pb]); J.nparts = nparts;
        return J;
      };
      auto resid_job = [&](const cfb_linear& lin, int e, size_t o_in, int ldin) {
        const int S = (e + 1) * d.chunk;
        cfb::Job J = make_job(lin, Bq * S);
        J.xkind = cfb::XK_F16; J.x = B.dptr<__half>(o_in); J.ldx = ldin;
        J.ekind = cfb::EK_RESID; J.out32 = B.dptr<float>(o_x32[2 * e + pb]);
        J.out16 = B.dptr<__half>(o_x16[2 * e + pb]); J.ldo = D;
        J.ostats = B.dptr<float2>(o_xs[2 * e + pb]); J.onparts = nparts;
        return J;
      };
      for (int l = 0; l < L; ++l) {
        std::vector<cfb::Job> js;
        for (int e = 0; e < E; ++e) {           // LN + self-attention in-projection
          const cfb_block& bl = d.experts[e].blocks[l];
          if (!lin_ok(bl.qkv, 3 * D, D)) return CFB_ERR_INVALID_ARG;
          cfb::Job J = ln_job(bl.qkv, e);
          J.ekind = cfb::EK_STORE; J.out32 = B.dptr<float>(o_qkv[e]); J.ldo = 3 * D;
          js.push_back(J);
        }
        add_phase(B, cfb::Phase{}, js); js.clear();
        add_attn(0);
        for (int e = 0; e < E; ++e) {           // out-projection + residual
          const cfb_block& bl = d.experts[e].blocks[l];
          if (!lin_ok(bl.self_out, D, D)) return CFB_ERR_INVALID_ARG;
          js.push_back(resid_job(bl.self_out, e, o_o[e], D));
        }
        add_phase(B, cfb::Phase{}, js); js.clear();
        for (int e = 0; e < E; ++e) {           // LN + cross-attention query projection
          const cfb_block& bl = d.experts[e].blocks[l];
          if (!lin_ok(bl.cross_q, D, D)) return CFB_ERR_INVALID_ARG;
          cfb::Job J = ln_job(bl.cross_q, e);
          J.ekind = cfb::EK_STORE; J.out32 = B.dptr<float>(o_qc[e]); J.ldo = D;
          js.push_back(J);
        }
        add_phase(B, cfb::Phase{}, js); js.clear();
        add_attn(E + l * E);
        for (int e = 0; e < E; ++e) {
          const cfb_block& bl = d.experts[e].blocks[l];
          if (!lin_ok(bl.cross_out, D, D)) return CFB_ERR_INVALID_ARG;
          js.push_back(resid_job(bl.cross_out, e, o_o[e], D));
        }
        add_phase(B, cfb::Phase{}, js); js.clear();
        for (int e = 0; e < E; ++e) {           // LN + FFN up + GELU
          const cfb_block& bl = d.experts[e].blocks[l];
          if (!lin_ok(bl.ffn_up, FM * D, D)) return CFB_ERR_INVALID_ARG;
          cfb::Job J = ln_job(bl.ffn_up, e);
          J.ekind = cfb::EK_GELU16; J.out16 = B.dptr<__half>(o_u[e]); J.ldo = FM * D;
          js.push_back(J);
        }
        add_phase(B, cfb::Phase{}, js); js.clear();
        for (int e = 0; e < E; ++e) {           // FFN down + residual
          const cfb_block& bl = d.experts[e].blocks[l];
          if (!lin_ok(bl.ffn_down, D, FM * D)) return CFB_ERR_INVALID_ARG;
          js.push_back(resid_job(bl.ffn_down, e, o_u[e], FM * D));
        }
        add_phase(B, cfb::Phase{}, js); js.clear();
      }
      std::vector<cfb::Job> js;                 // out_norm + out_proj, Euler, next inputs
      for (int e = 0; e < E; ++e) {
        const cfb_expert& ex = d.experts[e];
        const int S = (e + 1) * d.chunk;
        if (!lin_ok(ex.out_proj, D, D) || !ex.out_proj.bias) return CFB_ERR_INVALID_ARG;
        cfb::Job J = ln_job(ex.out_proj, e);
        J.rows = Bq * d.chunk; J.oR = J.rows;
        J.xR = Bq * S; J.xcopy = Bq * S;            // copy every row; the MMA picks the chunk's
        J.gin = d.chunk; J.gstride = S; J.goff = e * d.chunk;
        J.ekind = cfb::EK_EULER; J.e_idx = e; J.step = s; J.last_step = (s == T - 1);
        J.dt = 1.0f / (float)T;
        js.push_back(J);
      }
      add_phase(B, cfb::Phase{}, js);
    }
  }
  if (beam) {
    int fr = tree ? 1 : Wmax, base = 0, base_prev = 0;
    if (TPM) {   // pass A of the two-pass head: candidates for every depth from one head GEMM
      { cfb::Phase p{}; p.kind = cfb::PK_TPXA; ph.push_back(p); }
      {
        cfb::Job J = make_job(d.head, Bq * K);
        J.xkind = cfb::XK_F16; J.x = B.dptr<__half>(o_txa); J.ldx = D + rank;
        J.ekind = cfb::EK_HEAD; J.R = d.head.nout; J.rowoff = 0; J.topb = 1;
        J.bias = nullptr; J.colsum = nullptr; J.logits = B.dptr<float>(o_tlog);
        cfb::Phase p{};
        p.post = cfb::PO_PUBLISH; p.rows = Bq * K; p.topb = 1;
        add_phase(B, p, {J});
      }
      { cfb::Phase p{}; p.kind = cfb::PK_TPKEY; ph.push_back(p); }
      for (int pass = 1; pass < 4; ++pass) { cfb::Phase p{}; p.kind = cfb::PK_TPRAD; p.step = pass; ph.push_back(p); }
      { cfb::Phase p{}; p.kind = cfb::PK_TPCNT; ph.push_back(p); }
      { cfb::Phase p{}; p.kind = cfb::PK_TPSEL; ph.push_back(p); }
      { cfb::Phase p{}; p.kind = cfb::PK_TPGATH; ph.push_back(p); }
    }
    const int TB = tree ? r.tree_topb : r.width;
    for (int step = 1; step <= K; ++step) {
      const int rows = Bq * fr;
      const int nlive = std::min(step, order);
      {   // h = sum_j mask_j (W_j emb(lastp_j) + b_j) over the live offsets (CF_PATH_TRIM)
        // over the embedding rows the previous beam phase (or prep, at depth 1) gathered
        cfb::Job J = make_job(d.path_offsets, rows);
        J.Kt = nlive * D / 16;
        J.nkc = (J.Kt + cfb::kUnitK - 1) / cfb::kUnitK;
        J.xkind = cfb::XK_F16; J.x = B.dptr<__half>(o_pg); J.ldx = order * D;
        J.order = order; J.D = D; J.wrows = fr;
        J.ekind = cfb::EK_PATHH; J.bias = nullptr; J.colsum = nullptr;
        J.p0 = d.path_offset_bias; J.nlive = nlive;
        J.out16 = B.dptr<__half>(o_h16); J.ldo = D;
        J.ostats = B.dptr<float2>(o_hstat); J.onparts = nparts;
        cfb::Phase p{}; p.rows = rows; p.step = step;
        add_phase(B, p, {J});
      }
      {   // LayerNorm + Linear(D, 2D) + GELU
        cfb::Job J = make_job(d.path_up, rows);
        J.xkind = cfb::XK_F16; J.x = B.dptr<__half>(o_h16); J.ldx = D;
        J.ln = cfb::LN_PARTS; J.stats = B.dptr<float2>(o_hstat); J.nparts = nparts;
        J.ekind = cfb::EK_GELU16; J.out16 = B.dptr<__half>(o_mpath); J.ldo = P2;
        add_phase(B, cfb::Phase{}, {J});
      }
      {   // Linear(2D, D) + the flow hidden of this depth -> head input rows
        cfb::Job J = make_job(d.path_down, rows);
        J.xkind = cfb::XK_F16; J.x = B.dptr<__half>(o_mpath); J.ldx = P2;
        J.ekind = cfb::EK_HEADIN; J.out16 = B.dptr<__half>(o_xhead); J.ldo = D + rank;
        J.step = step; J.wrows = fr;
        add_phase(B, cfb::Phase{}, {J});
      }
      if (TPM) {   // pass B: every beam row against its own request's candidate rows only
        cfb_linear cl{B.dptr<void>(o_tchead), nullptr, nullptr, Bq * TPM, D + rank};
        cfb::Job J = make_job(cl, rows);
        J.xkind = cfb::XK_F16; J.x = B.dptr<__half>(o_xhead); J.ldx = D + rank;
        J.ekind = cfb::EK_HEAD; J.R = Bq * TPM; J.rowoff = 0; J.topb = TB;
        J.bias = nullptr; J.colsum = nullptr;
        J.cand = B.dptr<int>(o_tcd); J.cmask = TPM; J.wrows = fr;
        cfb::Phase p{};
        p.post = cfb::PO_PUBLISH; p.rows = rows; p.topb = TB;
        if (step == 1) p.last = cfb::kWeightsWritten;
        add_phase(B, p, {J});
      } else {   // shortlist head + markov bias with online LSE + top-k per CTA
        cfb::Job J = make_job(d.head, rows);
        J.xkind = cfb::XK_F16; J.x = B.dptr<__half>(o_xhead); J.ldx = D + rank;
        J.ekind = cfb::EK_HEAD; J.R = d.head.nout; J.rowoff = d.head_row0; J.topb = TB;
        J.bias = nullptr; J.colsum = nullptr;
        cfb::Phase p{};
        p.post = cfb::PO_PUBLISH; p.rows = rows; p.topb = TB;
        add_phase(B, p, {J});
      }
      if (r.ranks > 1) {   // merge this rank's CTA lists; the caller gathers them across ranks
        cfb::Phase p{};
        p.kind = cfb::PK_RMERGE; p.rows = rows; p.fr = fr; p.topb = TB;
        ph.push_back(p);
        B.segs.push_back((int)ph.size());
      }
      {   // merge the CTAs' lists, beam step, next depth's gather
        cfb::Phase p{};
        p.kind = cfb::PK_BEAM;
        p.post = tree ? cfb::PO_BEAM_TREE : cfb::PO_BEAM_CHAIN;
        p.rows = rows; p.step = step; p.fr = fr; p.keep = Wmax; p.topb = TB;
        p.base = base; p.base_prev = base_prev; p.last = (step == K);
        ph.push_back(p);
      }
      if (step < K) {   // the next depth's gathered rows, over the whole grid
        cfb::Phase g{};
        g.kind = cfb::PK_GATHER;
        g.fr = tree ? std::min(Wmax, fr * TB) : Wmax;
        g.step = step + 1;
        ph.push_back(g);
      }
      if (tree) {
        const int k = std::min(Wmax, fr * TB);
        base_prev = base; base += k; fr = k;
      }
    }
    B.P.N = base;
  }
  // shared-memory layout: accumulator hand-off slots (double-buffered when that still leaves a
  // deep ring), the epilogue's scratch (attention of one head of one request, merge ids), one
  // reduced tile and row statistics; the rest of the budget goes to the ring, each stage = a
  // 16 KiB weights unit + the unit's activation rows
  {
    int rows_max = 1, xrows_max = 1;
    for (const auto& j : B.jobs) { rows_max = std::max(rows_max, j.rows); xrows_max = std::max(xrows_max, std::max(j.rows, j.xcopy)); }
    const int ntb = (rows_max + 7) / 8;
    const int bucket = ntb <= 2 ? ntb : ntb <= 4 ? 4 : ntb <= 6 ? 6 : 8;
    B.P.maxnt = ntb <= 1 ? 1 : ntb <= 2 ? 2 : ntb <= 4 ? 4 : 8;
    const int RP = bucket * 8;
    // the accumulator staging tile of gathered-row jobs, [kTileRows][kAccCols + 1] fp32
    const size_t slot_bytes = ((size_t)cfb::kTileRows * (cfb::kAccCols + 1) * 4 + 127) / 128 * 128;
    // an activation half of a stage: the slot rows padded to the MMA's N granule (8), 128 B each
    const int xhalf = (xrows_max + 7) / 8 * 8 * 128;
    size_t scratch = (size_t)2 * cfb::kRowsMax * cfb::kTopMax * 4;
    if (flow) {
      const int hd = D / d.heads, Kmax = std::max(DL, C);
      scratch = std::max(scratch, (size_t)((DL + 2 * Kmax) * hd + DL * Kmax) * 4);
    }
    if (vae) {
      const int hd = D / B.vae->heads, S = B.vrows;
      scratch = std::max(scratch, (size_t)(3 * S * hd + S * S) * 4);
    }
    // a split tile's owner lists the other contributors (at most G) in the scratch
    scratch = std::max(scratch, (size_t)(G + 1) * 4);
    scratch = (scratch + 127) / 128 * 128;
    // the reduced tile [kTileRows][RP + 1]: an odd row stride, so that threads walking consecutive
    // features of one row (and the accumulator readout's 16 lanes) hit distinct banks
    const int RPs = RP + 1;
    const int red = cfb::kTileRows * RPs * 4, rowstat = cfb::kRowsMax * 8, misc = 64;
    const int desc = cfb::kDescBufs * (cfb::kPhaseSlot + cfb::kJobCache * (int)sizeof(cfb::Job));
    const int bars = (2 * cfb::kMaxStages + 5) * 8;
    const int stage_bytes = cfb::kUnitBytes + 2 * xhalf;     // a multiple of 1024: stages stay aligned
    const long fixed = (long)slot_bytes + scratch + red + rowstat + misc + bars + 512 +
                       2 * cfb::kTileRows * 4 + desc + 16 + 1024;
    const int nst = (int)std::min<long>(cfb::kMaxStages, (cfb::kSmemBudget - fixed) / stage_bytes);
    if (nst < 3) return CFB_ERR_UNSUPPORTED;
    const int nbuf = 2;                                        // TMEM accumulators
    cfb::SmemLayout& Lm = B.P.sm;
    Lm.nstages = nst; Lm.stage_bytes = stage_bytes; Lm.rows_pad = RPs; Lm.nbuf = nbuf; Lm.xhalf = xhalf;
    Lm.off_bar = nst * stage_bytes;
    Lm.off_slots = (Lm.off_bar + (2 * nst + 5) * 8 + 127) / 128 * 128;
    Lm.off_scratch = Lm.off_slots + (int)slot_bytes;
    Lm.off_red = Lm.off_scratch + (int)scratch;
    Lm.off_rowstat = Lm.off_red + red;
    Lm.off_tile = Lm.off_rowstat + rowstat;
    Lm.off_misc = Lm.off_tile + 2 * cfb::kTileRows * 4;
    Lm.off_desc = (Lm.off_misc + misc + 15) / 16 * 16;
    Lm.total = Lm.off_desc + desc + 1024;      // + the slack for aligning the base to 1024 bytes
  }
  if (B.too_big) return CFB_ERR_UNSUPPORTED;
  const size_t o_prof = profile ? A.take(ph.size() * (size_t)G * cfb::kProfSlots * 8) : 0;
  const size_t o_tilecnt = A.take((size_t)std::max(B.max_tiles, 1) * 4);
  B.off_phases = A.take(ph.size() * sizeof(cfb::Phase));
  B.off_jobs = A.take(std::max<size_t>(B.jobs.size(), 1) * sizeof(cfb::Job));
  B.off_attn = A.take(std::max<size_t>(at.size(), 1) * sizeof(cfb::AttnTask));
  *bytes = A.take(0);

  cfb::Plan& P = B.P;
  P.G = G; P.nphases = (int)ph.size(); P.mode = mode; P.B = Bq; P.D = D; P.DL = DL;
  P.n_experts = E; P.chunk = d.chunk; P.C = C; P.steps = d.steps; P.order = order; P.rank = rank;
  P.vocab = d.vocab; P.R = d.shortlist_rows; P.width = r.width; P.depth = r.depth;
  P.keep = r.tree_keep; P.topb = r.tree_topb; P.Wmax = Wmax;
  P.phases = B.dptr<cfb::Phase>(B.off_phases);
  P.jobs = B.dptr<cfb::Job>(B.off_jobs);
  P.attn = B.dptr<cfb::AttnTask>(B.off_attn);
  if (flow) {
    for (int e = 0; e < E; ++e) {
      cfb::ExpertRT& X = P.ex[e];
      for (int q = 0; q < 2; ++q) {
        X.x32[q] = B.dptr<float>(o_x32[2 * e + q]);
        X.x16[q] = B.dptr<__half>(o_x16[2 * e + q]);
        X.xstat[q] = B.dptr<float2>(o_xs[2 * e + q]);
      }
      X.S = (e + 1) * d.chunk; X.start = e * d.chunk;
      X.pos = d.experts[e].pos_emb; X.temb = d.experts[e].temb;
      // the Euler epilogue moves 8-column groups of these rows (and of pred) as 16-byte accesses
      if (!X.pos || !X.temb || ((reinterpret_cast<uintptr_t>(X.pos) | reinterpret_cast<uintptr_t>(X.temb) |
                                 reinterpret_cast<uintptr_t>(r.pred)) & 15))
        return CFB_ERR_INVALID_ARG;
    }
  }
  P.buf[CFB_BUF_PHASES] = const_cast<cfb::Phase*>(P.phases);
  P.buf_bytes[CFB_BUF_PHASES] = ph.size() * sizeof(cfb::Phase);
  if (profile) {
    P.prof = B.dptr<unsigned long long>(o_prof);
    P.buf[CFB_BUF_PROF] = P.prof; P.buf_bytes[CFB_BUF_PROF] = ph.size() * (size_t)G * cfb::kProfSlots * 8;
  }
  P.bar = B.dptr<unsigned>(o_bar); P.exitcnt = P.bar + 1;
  P.err = reinterpret_cast<int*>(P.bar + 3);
  P.tilecnt = B.dptr<unsigned>(o_tilecnt); P.ntilecnt = B.max_tiles;
  P.gpart = B.dptr<float>(o_gpart); P.hpart = B.dptr<float>(o_hpart);
  P.ctx = static_cast<const __half*>(r.ctx); P.z0 = static_cast<const __half*>(r.z0);
  P.pred = r.pred; P.ctxstat = B.dptr<float2>(o_ctxs); P.init_mode = r.init_mode;
  P.wait_ns = r.wait_budget_ns ? r.wait_budget_ns : cfb::kWaitBudgetNs;
  if (flow) P.ctx16 = B.dptr<__half>(o_ctx16);
  P.known0 = r.known0; P.tokens = r.tokens;
  if (vae) {
    P.vin = B.vin; P.vin32 = B.vdecode; P.vS = B.vrows; P.vDin = B.vae->in_dim;
    P.vin16 = B.dptr<__half>(o_vin16); P.vx32 = B.dptr<float>(o_vx32); P.vpos = B.vae->pos;
  }
  {
    auto expose = [&](int i, size_t off, size_t nbytes) { P.buf[i] = B.dptr<void>(off); P.buf_bytes[i] = nbytes; };
    if (beam) {
      expose(CFB_BUF_PATH_H16, o_h16, (size_t)rowsB * k128(D) * 2);
      expose(CFB_BUF_PATH_MID, o_mpath, (size_t)rowsB * k128(P2) * 2);
      expose(CFB_BUF_HEAD_IN, o_xhead, (size_t)rowsB * k128(D + rank) * 2);
      expose(CFB_BUF_LASTP, o_lastp, (size_t)rowsB * order * 8);
      expose(CFB_BUF_CUM, o_cum, (size_t)rowsB * 4);
    }
    if (flow) {
      const size_t rows1 = (size_t)Bq * d.chunk;
      expose(CFB_BUF_QKV0, o_qkv[0], rows1 * 3 * D * 4);
      expose(CFB_BUF_X32_0, o_x32[0], rows1 * D * 4);
      expose(CFB_BUF_KVC0, o_kvc[0], (size_t)d.layers * Bq * C * 2 * D * 4);
    }
  }
  if (beam) {
    P.lastp = B.dptr<int64_t>(o_lastp); P.cum = B.dptr<float>(o_cum);
    P.toks = B.dptr<int64_t>(o_toks); P.bps = B.dptr<int>(o_bps);
    P.shortlist = d.shortlist; P.markov_w1 = static_cast<const __half*>(d.markov_w1);
    P.xhead = B.dptr<__half>(o_xhead); P.ldxhead = D + rank;
    P.emb = static_cast<const __half*>(d.embed); P.pg = B.dptr<__half>(o_pg);
    P.tp_m = TPM; P.tp_n = TPM ? K : 0; P.tp_rs = (d.shortlist_rows + 3) / 4 * 4;
    if (TPM) {
      P.tp_head = static_cast<const uint4*>(d.head.w);
      P.txa = B.dptr<__half>(o_txa); P.tlog = B.dptr<float>(o_tlog); P.tkeys = B.dptr<unsigned>(o_tkeys);
      P.tcd = B.dptr<int>(o_tcd); P.tchead = B.dptr<uint4>(o_tchead);
      P.thist = B.dptr<unsigned>(o_thist); P.tcnt = B.dptr<int>(o_tcnt);
      P.buf[CFB_BUF_TP_CAND] = P.tcd; P.buf_bytes[CFB_BUF_TP_CAND] = (size_t)Bq * TPM * 4;
      P.buf[CFB_BUF_TP_CHEAD] = P.tchead;
      P.buf_bytes[CFB_BUF_TP_CHEAD] = ((size_t)Bq * TPM + 63) / 64 * 64 * (size_t)(D + rank) * 2;
    }
  }
  P.nranks = (beam && r.ranks > 1) ? r.ranks : 1;
  P.xloc = r.xloc; P.xall = r.xall;
  // launch segments: [0, s1), [s1, s2), ... [sk, nphases); the last boundary (after the final
  // depth's merge) leaves only the last beam phase in the final segment
  if ((int)B.segs.size() + 1 > cfb::kMaxSeg) return CFB_ERR_UNSUPPORTED;
  P.nseg = (int)B.segs.size() + 1;
  P.seg[0] = 0;
  for (size_t i = 0; i < B.segs.size(); ++i) P.seg[i + 1] = B.segs[i];
  P.seg[P.nseg] = (int)ph.size();
  return CFB_OK;
}

struct LaunchRecord { int G, phases, smem, pad; };
struct LaunchRec { void* ws; int G, smem, nseg, maxnt; bool prof; int seg[cfb::kMaxSeg + 1]; };
std::vector<LaunchRec> g_launch;     // launch shape of the plan last built in each workspace
using EngineFn = void (*)(const cfb::Plan*, int, int);
// the engine_kernel instantiation for plans whose widest job has `maxnt` 8-row n-tiles, with or
// without the per-phase profiling stamps
EngineFn engine_for(int maxnt, bool) {
  switch (maxnt) {
    case 1: return cfb::engine_kernel<1>;
    case 2: return cfb::engine_kernel<2>;
    case 4: return cfb::engine_kernel<4>;
    default: return cfb::engine_kernel<8>;
  }
}
int kernel_slot(int maxnt, bool) { return maxnt == 1 ? 0 : maxnt == 2 ? 1 : maxnt == 4 ? 2 : 3; }
void remember_launch(void* ws, const cfb::Plan& P, int smem) {
  LaunchRec r{ws, P.G, smem, P.nseg, P.maxnt, P.prof != nullptr, {}};
  for (int i = 0; i <= P.nseg; ++i) r.seg[i] = P.seg[i];
  for (auto& l : g_launch) if (l.ws == ws) { l = r; return; }
  g_launch.push_back(r);
}
// The kernel's dynamic shared-memory limit is a property of the function (per device), shared
// by every plan: raise it to what this plan needs, never lower it under another plan.
cfb_status ensure_smem_attr(int maxnt, bool prof, int smem) {
  static std::mutex mu;
  static int attr[64][8] = {};
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_fail(e, "get device");
  const int k = kernel_slot(maxnt, prof);
  std::lock_guard<std::mutex> lock(mu);
  if (dev >= 0 && dev < 64 && attr[dev][k] >= smem) return CFB_OK;
  e = cudaFuncSetAttribute(engine_for(maxnt, prof), cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  if (e != cudaSuccess) return cuda_fail(e, "smem attribute");
  if (dev >= 0 && dev < 64) attr[dev][k] = smem;
  return CFB_OK;
}

// the launch record of workspace ws: the host copy, else read back from the device plan
cfb_status launch_rec(void* ws, LaunchRec& out) {
  for (auto& l : g_launch) if (l.ws == ws) { out = l; return CFB_OK; }
  cfb::Plan P;
  cudaError_t e = cudaMemcpy(&P, static_cast<uint8_t*>(ws) + kOffPlan, sizeof(P), cudaMemcpyDeviceToHost);
  if (e != cudaSuccess) return cuda_fail(e, "read plan record");
  if (P.nseg < 1 || P.nseg > cfb::kMaxSeg) return CFB_ERR_INVALID_ARG;
  remember_launch(ws, P, P.sm.total);
  for (auto& l : g_launch) if (l.ws == ws) { out = l; return CFB_OK; }
  return CFB_ERR_INVALID_ARG;
}

}  // namespace

extern "C" {

const char* cfb_last_cuda_error(void) { return g_cuda_err; }
int cfb_abi_version(void) { return CFB_ABI_VERSION; }

cfb_status cfb_plan_workspace(const cfb_drafter* d, const cfb_run* r, size_t* bytes) {
  if (!d || !r || !bytes) return CFB_ERR_INVALID_ARG;
  Builder B; B.d = d; B.r = r; B.base = nullptr;
  return lower(B, bytes);
}

}  // extern "C"

namespace {
// Lower B into the workspace and record the launch shape (cfb_plan_build, cfb_vae_plan_build).
cfb_status build_into(Builder& B, void* ws, size_t bytes) {
  size_t need = 0;
  cfb_status st = lower(B, &need);
  if (st != CFB_OK) return st;
  if (need > bytes) return CFB_ERR_WORKSPACE;
  cudaError_t e;
  const int smem = B.P.sm.total;
  const bool prof = B.P.prof != nullptr;
  if ((st = ensure_smem_attr(B.P.maxnt, prof, smem)) != CFB_OK) return st;
  int per_sm = 0, dev = 0, sms = 0;
  if ((e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, engine_for(B.P.maxnt, prof), cfb::kThreads, smem)) !=
      cudaSuccess)
    return cuda_fail(e, "occupancy");
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  if (per_sm < 1 || B.P.G > per_sm * sms) return CFB_ERR_COOP_LAUNCH;
  if ((e = cudaMemcpy(B.base + B.off_phases, B.phases.data(), B.phases.size() * sizeof(cfb::Phase),
                      cudaMemcpyHostToDevice)) != cudaSuccess) return cuda_fail(e, "copy phases");
  if (!B.jobs.empty() &&
      (e = cudaMemcpy(B.base + B.off_jobs, B.jobs.data(), B.jobs.size() * sizeof(cfb::Job),
                      cudaMemcpyHostToDevice)) != cudaSuccess) return cuda_fail(e, "copy jobs");
  if (!B.attn.empty() &&
      (e = cudaMemcpy(B.base + B.off_attn, B.attn.data(), B.attn.size() * sizeof(cfb::AttnTask),
                      cudaMemcpyHostToDevice)) != cudaSuccess) return cuda_fail(e, "copy attention tasks");
  if ((e = cudaMemcpy(B.base + kOffPlan, &B.P, sizeof(cfb::Plan), cudaMemcpyHostToDevice)) != cudaSuccess)
    return cuda_fail(e, "copy plan");
  const size_t ob = off_barrier();
  if ((e = cudaMemset(B.base + ob, 0, 64)) != cudaSuccess) return cuda_fail(e, "zero barrier");
  LaunchRecord h{B.P.G, B.P.nphases, smem, B.P.sm.nstages};
  if ((e = cudaMemcpy(B.base + ob + 32, &h, sizeof(h), cudaMemcpyHostToDevice)) != cudaSuccess)
    return cuda_fail(e, "copy launch record");
  if ((e = cudaDeviceSynchronize()) != cudaSuccess) return cuda_fail(e, "plan build sync");
  remember_launch(ws, B.P, smem);
  return CFB_OK;
}

// The stand-in drafter / run of a VAE side plan: D = the VAE width, one "expert" of `rows`
// rows so that the shared validation holds, the output bound as pred.
void vae_standins(const cfb_vae_side* v, int batch, int rows, void* out, cfb_drafter& d, cfb_run& r) {
  d = cfb_drafter{};
  r = cfb_run{};
  d.hidden = v->width; d.heads = v->heads; d.layers = v->layers; d.steps = 1;
  d.draft_len = rows; d.chunk = rows; d.ctx_rows = rows; d.n_experts = 1;
  r.mode = cfb::kModeVae; r.batch = batch; r.pred = static_cast<float*>(out);
}
}  // namespace

extern "C" {

cfb_status cfb_plan_build(const cfb_drafter* d, const cfb_run* r, void* ws, size_t bytes) {
  if (!d || !r || !ws) return CFB_ERR_INVALID_ARG;
  if (reinterpret_cast<uintptr_t>(ws) % 256) return CFB_ERR_INVALID_ARG;
  Builder B; B.d = d; B.r = r; B.base = static_cast<uint8_t*>(ws);
  return build_into(B, ws, bytes);
}

cfb_status cfb_vae_plan_workspace(const cfb_vae_side* v, int batch, int rows, int decode, size_t* bytes) {
  if (!v || !bytes || batch <= 0 || rows <= 0) return CFB_ERR_INVALID_ARG;
  cfb_drafter d; cfb_run r;
  void* any = reinterpret_cast<void*>(256);           // sizing pass: any non-null I/O address
  vae_standins(v, batch, rows, any, d, r);
  Builder B; B.d = &d; B.r = &r; B.base = nullptr;
  B.vae = v; B.vrows = rows; B.vdecode = decode != 0; B.vin = any; B.vout = any;
  return lower(B, bytes);
}

cfb_status cfb_vae_plan_build(const cfb_vae_side* v, int batch, int rows, int decode, const void* in, void* out,
                              void* ws, size_t bytes) {
  if (!v || !ws || !in || !out || batch <= 0 || rows <= 0) return CFB_ERR_INVALID_ARG;
  if (reinterpret_cast<uintptr_t>(ws) % 256) return CFB_ERR_INVALID_ARG;
  cfb_drafter d; cfb_run r;
  vae_standins(v, batch, rows, out, d, r);
  Builder B; B.d = &d; B.r = &r; B.base = static_cast<uint8_t*>(ws);
  B.vae = v; B.vrows = rows; B.vdecode = decode != 0; B.vin = in; B.vout = out;
  return build_into(B, ws, bytes);
}

cfb_status cfb_plan_info(void* ws, int* grid, int* threads, int* smem, int* phases) {
  if (!ws) return CFB_ERR_INVALID_ARG;
  LaunchRecord h{};
  cudaError_t e = cudaMemcpy(&h, static_cast<uint8_t*>(ws) + off_barrier() + 32, sizeof(h),
                             cudaMemcpyDeviceToHost);
  if (e != cudaSuccess) return cuda_fail(e, "read launch record");
  if (grid) *grid = h.G;
  if (threads) *threads = cfb::kThreads;
  if (smem) *smem = h.smem;
  if (phases) *phases = h.phases;
  return CFB_OK;
}

static cfb_status launch_range(void* ws, const LaunchRec& L, int p0, int p1, void* stream) {
  const cfb_status st = ensure_smem_attr(L.maxnt, L.prof, L.smem);
  if (st != CFB_OK) return st;
  const cfb::Plan* Pd = reinterpret_cast<const cfb::Plan*>(static_cast<uint8_t*>(ws) + kOffPlan);
  void* args[] = {(void*)&Pd, (void*)&p0, (void*)&p1};
  cudaError_t e = cudaLaunchCooperativeKernel((const void*)engine_for(L.maxnt, L.prof), dim3(L.G), dim3(cfb::kThreads),
                                              args, (size_t)L.smem, static_cast<cudaStream_t>(stream));
  if (e == cudaErrorCooperativeLaunchTooLarge) return CFB_ERR_COOP_LAUNCH;
  if (e != cudaSuccess) return cuda_fail(e, "engine launch");
  return CFB_OK;
}

cfb_status cfb_plan_run(void* ws, void* stream) {
  if (!ws) return CFB_ERR_INVALID_ARG;
  LaunchRec L;
  cfb_status st = launch_rec(ws, L);
  if (st != CFB_OK) return st;
  if (L.nseg != 1) return CFB_ERR_INVALID_ARG;     // sharded heads run segment by segment
  return launch_range(ws, L, 0, L.seg[1], stream);
}

cfb_status cfb_plan_segments(void* ws, int* nseg) {
  if (!ws || !nseg) return CFB_ERR_INVALID_ARG;
  LaunchRec L;
  cfb_status st = launch_rec(ws, L);
  if (st != CFB_OK) return st;
  *nseg = L.nseg;
  return CFB_OK;
}

cfb_status cfb_plan_run_segment(void* ws, int seg, void* stream) {
  if (!ws) return CFB_ERR_INVALID_ARG;
  LaunchRec L;
  cfb_status st = launch_rec(ws, L);
  if (st != CFB_OK) return st;
  if (seg < 0 || seg >= L.nseg) return CFB_ERR_INVALID_ARG;
  return launch_range(ws, L, L.seg[seg], L.seg[seg + 1], stream);
}

cfb_status cfb_plan_buffer(void* ws, int which, void** ptr, size_t* bytes) {
  if (!ws || !ptr || which < 0 || which >= 16) return CFB_ERR_INVALID_ARG;
  cfb::Plan P;
  cudaError_t e = cudaMemcpy(&P, static_cast<uint8_t*>(ws) + kOffPlan, sizeof(P), cudaMemcpyDeviceToHost);
  if (e != cudaSuccess) return cuda_fail(e, "read plan record");
  *ptr = P.buf[which];
  if (bytes) *bytes = P.buf_bytes[which];
  return P.buf[which] ? CFB_OK : CFB_ERR_INVALID_ARG;
}

cfb_status cfb_plan_error(void* ws, int* device_error) {
  if (!ws || !device_error) return CFB_ERR_INVALID_ARG;
  int v = 0;
  cudaError_t e = cudaMemcpy(&v, static_cast<uint8_t*>(ws) + off_barrier() + 12, sizeof(int),
                             cudaMemcpyDeviceToHost);
  if (e != cudaSuccess) return cuda_fail(e, "read error word");
  *device_error = v;
  return v == 0 ? CFB_OK : CFB_ERR_DEVICE_TIMEOUT;
}

}  // extern "C"
