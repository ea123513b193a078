/*
 * cfb.h -- C ABI of libcfb.so, the sm_100a drafting engine of chain_flow_b200.
 *
 * Plain C: device pointers, sizes and a cudaStream_t passed as void*. No torch types.
 * Every buffer (weights, inputs, outputs, workspace) is allocated by the CALLER; the library
 * allocates nothing per call.
 *
 * Reference interfaces replaced (paths relative to the reference checkout):
 *   src/chain_flow/csrc/fused_block.cu:784-862  cf_fused_block.{expert, cross_kv, max_grid}
 *       -> cfb_plan_workspace / cfb_plan_build / cfb_plan_run (the whole integrator, both
 *          chunk experts, all Euler steps, cross-K/V hoist, in one persistent launch)
 *   src/chain_flow/cuda_block.py:266-311 (weight packing)  -> cfb_pack_linear / cfb_fold_bias
 *   src/chain_flow/drafters/chunked_flow.py:230-234, 313-321 (time_mlp at tau = s/T)
 *                                                       -> cfb_time_embed
 *   src/chain_flow/vllm_plugin/flow_proposer.py:1188-1269 (_beam_chains) and :1273-1332
 *       (_beam_tree), :1021-1028 (_head/_bias/_map), drafters/tree_flow.py:434-450
 *       (_residual_from_lastp)                        -> CFB_MODE_CHAIN / CFB_MODE_TREE plans
 *   src/chain_flow/kernels/tree_scan.py:43-78 (tree_gated_delta_scan) and the fork's
 *       tree_gdn_verify.cu gdn_verify_kernel (patch:4401-4562) -> cfb_tree_gdn
 */
#ifndef CFB_H_
#define CFB_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define CFB_ABI_VERSION 5

typedef enum cfb_status {
  CFB_OK = 0,
  CFB_ERR_INVALID_ARG = 1,     /* null pointer, negative size, misaligned buffer */
  CFB_ERR_UNSUPPORTED = 2,     /* shape outside what the kernels are built for */
  CFB_ERR_WORKSPACE = 3,       /* workspace smaller than cfb_plan_workspace() asked for */
  CFB_ERR_CUDA = 4,            /* a CUDA runtime call failed (cfb_last_cuda_error() says which) */
  CFB_ERR_COOP_LAUNCH = 5,     /* the persistent grid cannot be co-resident on this device */
  CFB_ERR_DEVICE_TIMEOUT = 6   /* a bounded device-side wait expired; outputs are invalid */
} cfb_status;

/* ---- packed weights --------------------------------------------------------------------
 * A packed linear holds W (fp16, [nout, k] like nn.Linear.weight) in the engine's streaming
 * layout: rows padded to a multiple of 64 and k to a multiple of 64, then
 * [nout/64][k/64][64 rows][128 B]: each 128-byte row holds 64 consecutive k of one output row,
 * its 16-byte chunks XOR-swizzled by (row & 7), so every [64 x 64] block (8 KiB) is the
 * shared-memory image of a K-major, 128-byte-swizzled tcgen05 operand. A streamed unit is two
 * consecutive blocks (128 k) of one 64-row tile: 16 KiB, contiguous. A LayerNorm in front of the linear is folded
 * in: W' = fp16(W diag(gamma)), bias' = b + W beta and colsum = sum_k W'[:, k]; the engine then
 * computes y = (W' x - mean * colsum) * rstd + bias' from the un-normalised fp16 input. */
typedef struct cfb_linear {
  const void*  w;       /* packed fp16, cfb_packed_bytes(nout, k) bytes, 16-byte aligned */
  const float* bias;    /* fp32 [nout] or NULL */
  const float* colsum;  /* fp32 [nout] when a LayerNorm is folded in, else NULL */
  int nout;
  int k;                /* multiple of 16 */
} cfb_linear;

/* one HiddenKVFlowBlock (reference drafters/chunked_flow.py:168-202) */
typedef struct cfb_block {
  cfb_linear qkv;        /* self_attn.in_proj, self_norm folded          [3D, D] */
  cfb_linear self_out;   /* self_attn.out_proj                           [D, D]  */
  cfb_linear cross_q;    /* cross_attn.in_proj rows [0,D), cross_norm folded   [D, D]  */
  cfb_linear cross_kv;   /* cross_attn.in_proj rows [D,3D), context_norm folded [2D, D] */
  cfb_linear cross_out;  /* cross_attn.out_proj                          [D, D]  */
  cfb_linear ffn_up;     /* ffn.1, ffn.0 (LayerNorm) folded              [FM*D, D] */
  cfb_linear ffn_down;   /* ffn.4                                        [D, FM*D] */
} cfb_block;

/* one HiddenKVFlowExpert (reference drafters/chunked_flow.py:205-414) */
typedef struct cfb_expert {
  const float* pos_emb;     /* fp32 [draft_len, D]: position_embedding.weight (16-byte aligned) */
  const float* temb;        /* fp32 [steps, D]: time_mlp(s / steps), from cfb_time_embed (16-byte aligned) */
  cfb_linear out_proj;      /* out_proj, out_norm folded [D, D] */
  const cfb_block* blocks;  /* HOST array [layers] */
} cfb_expert;

typedef struct cfb_drafter {
  int hidden;          /* D == target hidden size (TreeFlowDrafter, tree_flow.py:113-114) */
  int heads;           /* attention heads (8) */
  int layers;          /* blocks per expert */
  int steps;           /* Euler steps */
  int draft_len;       /* flow positions (draft_length) */
  int chunk;           /* rows per chunk expert (chunk_size) */
  int ctx_rows;        /* context window rows (context_size) */
  int n_experts;       /* draft_len / chunk */
  const cfb_expert* experts;   /* HOST array [n_experts] */
  /* path head, markov bias and shortlist head (the beam) */
  int path_order;
  int markov_rank;
  int vocab;
  int shortlist_rows;          /* R */
  const void* embed;           /* fp16 [vocab, D] target input embeddings */
  cfb_linear path_offsets;     /* [D, order*D]: offset_proj.j.weight side by side; bias NULL */
  const float* path_offset_bias; /* fp32 [order, D] */
  cfb_linear path_up;          /* path_head.mlp.0, path_head.norm folded [2D, D] */
  cfb_linear path_down;        /* path_head.mlp.3 [D, 2D] */
  const void* markov_w1;       /* fp16 [vocab, rank] */
  cfb_linear head;             /* [R, D + rank] = [lm_head.weight[sl] | markov.w2.weight[sl]],
                                  or rows [head_row0, head_row0 + head.nout) of it (a row shard) */
  const int64_t* shortlist;    /* int64 [R] global token ids (sorted, unique) */
  int head_row0;               /* first shortlist row `head` holds: 0 unless the head is sharded */
} cfb_drafter;

typedef enum cfb_mode {
  CFB_MODE_FLOW = 0,        /* integrate only:  ctx, z0 -> pred */
  CFB_MODE_CHAIN = 1,       /* flow + chain beam: ctx, z0, known0 -> tokens [B, depth] */
  CFB_MODE_TREE = 2,        /* flow + tree beam:  ctx, z0, known0 -> tokens [B, 2N] */
  CFB_MODE_BEAM_CHAIN = 3,  /* chain beam over a given pred */
  CFB_MODE_BEAM_TREE = 4    /* tree beam over a given pred */
} cfb_mode;

/* initial latents z0 of the flow (reference TreeFlowDrafter.init_latents, tree_flow.py:150-161) */
typedef enum cfb_init {
  CFB_INIT_GIVEN = 0,        /* z0 supplied by the caller (init_mode='noise': the caller draws it) */
  CFB_INIT_REPEAT_LAST = 1,  /* every position = the last context row */
  CFB_INIT_DELTA = 2         /* position i = last + (i+1) * (last - previous context row) */
} cfb_init;

typedef struct cfb_run {
  int mode;            /* cfb_mode */
  int init_mode;       /* cfb_init */
  int batch;           /* requests B */
  int width;           /* chain beam width (CF_WIDTH, reference flow_proposer.py:374) */
  int depth;           /* chain: emitted tokens K; tree: levels (CF_TREE_DEPTH) */
  int tree_keep;       /* CF_TREE_KEEP */
  int tree_topb;       /* CF_TREE_TOPB */
  int grid;            /* persistent CTAs; 0 = one per SM */
  int flags;           /* CFB_RUN_PROFILE: record per-phase %globaltimer stamps (CFB_BUF_PROF) */
  /* device I/O, bound at cfb_plan_build time (graph-stable addresses) */
  const void* ctx;     /* fp16 [B, ctx_rows, D] */
  const void* z0;      /* fp16 [B, draft_len, D] initial latents (CFB_INIT_GIVEN only) */
  const int64_t* known0;  /* int64 [B] committed token per request */
  float* pred;         /* fp32 [B, draft_len, D]: output of the flow, input of BEAM_* modes (16-byte
                          aligned in the flow modes) */
  int64_t* tokens;     /* int64 chain [B, depth]; tree [B, 2N] (N tokens, then N parents) */
  /* Row-sharded shortlist head across `ranks` GPUs (ranks > 1): every rank runs the same
   * requests with the same inputs; the flow is computed on every rank, the head only over this
   * rank's rows (cfb_drafter.head_row0 / head.nout). Per beam depth the plan merges its CTAs'
   * lists into xloc [CFB_XROWS][CFB_XFLOATS] fp32 (max, sumexp, top-k values, top-k ids as
   * float bits, per beam row), ends a segment, and expects the caller to gather every rank's
   * xloc, in rank order, into xall [ranks][CFB_XROWS][CFB_XFLOATS] before the next segment. */
  int ranks;           /* 0 or 1: no sharding */
  int rank;
  float* xloc;
  const float* xall;
  /* The two-pass candidate head (reference CF_TWOPASS_M with CF_TWOPASS_SHARED=1 and
   * CF_TWOPASS_SEED=0, flow_proposer.py:1142-1184); 0 = the one-pass head. Pass A scores the
   * marginal hiddens of depths 1..K against the whole shortlist head in one GEMM and keeps, per
   * request, the twopass_m shortlist rows with the best log-prob over those depths; every depth
   * then rescores its beam rows against those rows only (log-softmax over the candidates).
   * Engine plans on one GPU (ranks <= 1); 0 < twopass_m < shortlist_rows. */
  int twopass_m;
  /* Budget in ns of the waits that order the work of a draft (0 = the default, 1 s): the grid
   * barrier between the phases of an engine plan, and in the wide plan's GEMMs the producer's
   * wait for a free ring stage and the MMA issuer's wait for a loaded one. A wait that outlasts it
   * ends the run with the plan's device error word set (cfb_plan_error / cfb_wide_error), and
   * the run after a rebuild is clean. A budget below the default is checked at every poll, so a
   * tiny one (1 ns) makes those waits expire on purpose: that is how the failure path is
   * tested. Waits for copies already in flight (before a CTA may exit) always get the default. */
  uint64_t wait_budget_ns;
} cfb_run;

#define CFB_XROWS 64
#define CFB_XFLOATS 18

int cfb_abi_version(void);
const char* cfb_last_cuda_error(void);

/* bytes of a packed [nout, k] linear */
size_t cfb_packed_bytes(int nout, int k);

/* Pack fp16 W[rows[i] or i, :k] (row stride ldw elements) into columns [kofs, kofs+k) of a
 * packed [nout, ktotal] buffer, scaling column j by gamma[j] when gamma != NULL. */
cfb_status cfb_pack_linear(const void* w, int64_t ldw, const int64_t* rows, int nout, int k,
                           const float* gamma, void* dst, int ktotal, int kofs, void* stream);

/* LayerNorm folding for one linear W [nout, k] (fp16, row stride ldw):
 *   bias_out[i]   = (bias ? bias[i] : 0) + sum_j W[i, j] * beta[j]
 *   colsum_out[i] = sum_j fp16(W[i, j] * gamma[j])       (colsum_out may be NULL) */
cfb_status cfb_fold_bias(const void* w, int64_t ldw, int nout, int k, const float* gamma,
                         const float* beta, const float* bias, float* bias_out, float* colsum_out,
                         void* stream);

/* out[s, :] = W2 silu(w1 * (s/steps) + b1) + b2 for s in [0, steps): the time embedding of
 * every Euler step (the reference evaluates time_mlp at the same tau for every row) */
cfb_status cfb_time_embed(const float* w1, const float* b1, const void* w2_f16, const float* b2,
                          int D, int steps, float* out, void* stream);

/* Plan = phase table + scratch for one (drafter, run) pair, laid out in a caller buffer. */
cfb_status cfb_plan_workspace(const cfb_drafter* d, const cfb_run* r, size_t* bytes);
/* Synchronous set-up: validates shapes, writes the phase table into ws, zeroes counters. */
cfb_status cfb_plan_build(const cfb_drafter* d, const cfb_run* r, void* ws, size_t bytes);
/* Launch the persistent kernel on `stream` (no allocation, no host synchronisation) for the
 * whole draft. Plans with a sharded head (cfb_run.ranks > 1) run segment by segment instead. */
cfb_status cfb_plan_run(void* ws, void* stream);
/* Segments of a built plan: 1, or K + 1 for a sharded head (the caller gathers xloc into xall
 * after every segment but the last). cfb_plan_run_segment launches one of them. */
cfb_status cfb_plan_segments(void* ws, int* nseg);
cfb_status cfb_plan_run_segment(void* ws, int seg, void* stream);
/* Synchronous: the plan's device error word: 0 while every run so far completed, else the code
 * of the first failure (a bounded device-side wait that expired). The word is sticky: once it
 * is set, later runs of the plan return at once without touching the outputs, until
 * cfb_plan_build rebuilds the plan. */
cfb_status cfb_plan_error(void* ws, int* device_error);
/* Launch parameters the plan resolved (grid CTAs, threads, dynamic smem bytes, phases). */
cfb_status cfb_plan_info(void* ws, int* grid, int* threads, int* smem, int* phases);

/* Device address and size of one intermediate buffer of a built plan (stage-by-stage checks).
 * fp16 activation buffers are tiled: for R rows and K columns (K padded up to a multiple of 128),
 * element (r, k) is at ((k >> 6) * R + r) * 64 + ((((k & 63) >> 3) ^ (r & 7)) << 3) + (k & 7): each
 * 64-column slice of all rows is contiguous, one 128-byte row per activation row with its 16-byte
 * chunks XOR-swizzled by (r & 7) (the tensor cores' K-major 128-byte-swizzled operand image).
 * CFB_BUF_PATH_H16   fp16 tiled [rows, D]     path offsets sum h (rows = B * frontier width)
 * CFB_BUF_PATH_MID   fp16 tiled [rows, 2D]    gelu(LN(h) W_up^T + b)
 * CFB_BUF_HEAD_IN    fp16 tiled [rows, D + r] [pred + residual | markov w1 row], the head input
 * CFB_BUF_LASTP      int64 [rows, order] beam paths (last `order` tokens, -1 = none)
 * CFB_BUF_CUM        fp32 [rows]         beam cumulative log-probs
 * CFB_BUF_QKV0       fp32 [B*chunk, 3D]  expert 0 self-attention in-projection output
 * CFB_BUF_X32_0      fp32 [B*chunk, D]   expert 0 residual stream (even Euler steps)
 * CFB_BUF_KVC0       fp32 [L, B*ctx, 2D] expert 0 cross-attention K/V of every block
 * Values hold what the last completed run left there. */
#define CFB_RUN_PROFILE 1
/* CFB_BUF_PROF        uint64 [phases, grid, 20] per CTA, %globaltimer ns: [0] phase start,
 *                     [1] work done, [2] grid barrier passed, [3] MMA warps waiting for data,
 *                     [4] MMA warps waiting for a free accumulator slot, [5] epilogue waiting for
 *                     partials, [6] epilogue done, [7] activation copies all issued, [8] weight
 *                     producer waiting for a free ring slot, [9] weight units all issued,
 *                     [10] / [11] the MMA warps' first / last unit of the phase ready (0 if
 *                     the CTA had no unit); for the epilogue's last tile of the phase: [12]
 *                     partials ready, [13] split-tile counter updated, [14] split-tile partials
 *                     summed (0 if not applicable), [15] tile finished; beam phases, in the
 *                     CTAs that own a request: [16] lists merged, [17] beam step done, [18] next
 *                     depth's rows gathered; [19] epilogue: the last job's row statistics
 *                     loaded (GEMM phases); written only by runs of plans built
 *                     with CFB_RUN_PROFILE */
enum { CFB_BUF_PROF = 8 };
/* CFB_BUF_PHASES      int32 [phases, 15] the phase table: [0] kind (0 prep, 1 GEMM, 2 attention,
 *                     3 beam, 4 rank merge, 5 next depth's path-row gather, 6-8 the two-pass
 *                     head's pass-A input, candidate selection and candidate-row gather), [1..5] first job, jobs, units, tiles, whole-tile flag,
 *                     [6] post-op (0 none, 1 chain beam, 2 tree beam, 3 head lists published:
 *                     the shortlist head GEMM of a beam depth), [7..14] step, rows, frontier,
 *                     kept beams, top list length, node base, previous node base, last-depth
 *                     flag. Read-only for the caller. */
enum { CFB_BUF_PHASES = 9 };
/* CFB_BUF_TP_CAND     int32 [B, twopass_m]: the two-pass head's candidate shortlist rows per
 *                     request, ascending (plans built with twopass_m > 0). */
enum { CFB_BUF_TP_CAND = 10 };
/* CFB_BUF_TP_CHEAD    the candidates' head rows [lm_head[sl] | markov.w2[sl]] of CFB_BUF_TP_CAND,
 *                     request-major, packed like cfb_pack_linear ([B * twopass_m, D + rank]). */
enum { CFB_BUF_TP_CHEAD = 11 };
enum { CFB_BUF_PATH_H16 = 0, CFB_BUF_PATH_MID = 1, CFB_BUF_HEAD_IN = 2, CFB_BUF_LASTP = 3,
       CFB_BUF_CUM = 4, CFB_BUF_QKV0 = 5, CFB_BUF_X32_0 = 6, CFB_BUF_KVC0 = 7 };
cfb_status cfb_plan_buffer(void* ws, int which, void** ptr, size_t* bytes);

/* Tree-aware Gated-DeltaNet verification over B independent trees of N nodes.
 * q,k [B,N,H,Dk] fp16; v [B,N,H,Dv] fp16; g (log decay), beta [B,N,H] fp32;
 * parent [B,N] int32 (parent < child; -1 = root, reads init; a node whose parent is neither
 * -1 nor an earlier node gets NaN output and state, as do its descendants, and the bad index is
 * never dereferenced); init [B,H,Dk,Dv] fp32;
 * out o [B,N,H,Dv] fp32; states [B,N,H,Dk,Dv] fp32 (every node's state; also where a child
 * reads its parent's state, so it is required).
 * use_l2norm: q,k <- x / (||x|| + 1e-6); q is scaled by Dk**-0.5.
 * Launches whose node-by-node grid would have fewer (request, head, 32-column) blocks than the
 * device has SMs run path-parallel: every node
 * walks its ancestor chain from init with the same per-node arithmetic; larger ones run node by
 * node. Both write the same states and outputs.
 * Supported: Dk == 128; Dv a multiple of 32; N <= 64 nodes per tree. */
cfb_status cfb_tree_gdn(const void* q, const void* k, const void* v, const float* g,
                        const float* beta, const int32_t* parent, const float* init,
                        float* o, float* states, int B, int N, int H, int Dk, int Dv,
                        int use_l2norm, void* stream);

/* The in-engine tree GDN verify (the contract of the reference's vLLM-patch kernel,
 * src/chain_flow/patches/vllm-0.25.1-chain-flow-tree.patch:4401-4562 / gdn_verify :4606): every
 * query row t re-walks its ancestor chain n = chain[t * chain_stride + kk], kk = depth[t] .. 0,
 * from state slot init_slot[t]:
 *   S <- S * exp(-exp(A_log[hv]) * softplus(a[n, hv] + dt_bias[hv]))   (softplus(x) = x above 20)
 *   S <- S + sigmoid(b[n, hv]) * (v[n, hv] - S kn) (x) kn,   kn = k[n, h] * rsqrt(|k[n, h]|^2 + 1e-6)
 * then o[t, hv] = S (q[t, h] * rsqrt(|q[t, h]|^2 + 1e-6) * scale) (write_out) and
 * state[out_slot[t], hv] = S (write_state), h = hv / (HV / H).
 * q, k [*, H, K] and v, o [*, HV, V] fp16 (qkv_dtype 1) or bf16 (2); a, b [*, HV] and A_log,
 * dt_bias [HV] of dtype code 0 (fp32), 1 (fp16) or 2 (bf16); state fp32 [slots, HV, V, K] with
 * slot stride slot_stride floats; chain, depth, out_slot, init_slot, rows int32; rows (may be
 * NULL) selects the T_rows query rows. Out slots must not be read as init slots by other rows
 * of the same call. A row whose depth does not fit its chain row (depth < 0 or >= chain_stride)
 * gets NaN output and state. The chain entries chain[t, 0 .. depth[t]] themselves are used as row
 * indices of k, v, a and b as given (the call has no row count to check them against). Supported:
 * K == 128, V a multiple of 32, HV a multiple of H, chain_stride <= 16. */
cfb_status cfb_tree_gdn_verify(const void* A_log, int A_log_dtype, const void* dt_bias,
                               int dt_bias_dtype, const void* a, int a_dtype, const void* b,
                               int b_dtype, const void* q, const void* k, const void* v, void* o,
                               int qkv_dtype, float* state, int64_t slot_stride,
                               const int32_t* chain, int chain_stride, const int32_t* depth,
                               const int32_t* out_slot, const int32_t* init_slot,
                               const int32_t* rows, float scale, int T_rows, int H, int HV, int K,
                               int V, int write_out, int write_state, void* stream);

/* The shared-root factorisation of the in-engine tree GDN verify (the contract of the reference
 * fork's gdn_factor, src/chain_flow/patches/vllm-0.25.1-chain-flow-tree.patch:4664-5094): the
 * outputs o of cfb_tree_gdn_verify, for S requests whose rows [row_start[s], +row_count[s]) all
 * start from the one state slot init_slot[row_start[s]], computed without reading or writing any
 * per-node state: every update is rank 1, so a node's state is the root state decayed plus one
 * rank-1 term per ancestor, and the root state is only used through H k and H q. The root state is
 * read once per (request, head). chain rows hold GLOBAL row ids (chain[t, 0] = t, chain[t, j] the
 * j-th ancestor, j <= depth[t]); a row whose chain leaves its request, or whose depth does not fit
 * the chain row, gets NaN. Other arguments as cfb_tree_gdn_verify. Supported: K == 128, V a multiple
 * of 32, row_count <= n_max <= 64, chain_stride <= 16. No state is written: the state that
 * survives verification (the accepted leaf's) is materialised afterwards with
 * cfb_tree_gdn_verify(write_out = 0, rows = the leaf). */
cfb_status cfb_tree_gdn_factor(const void* A_log, int A_log_dtype, const void* dt_bias,
                               int dt_bias_dtype, const void* a, int a_dtype, const void* b,
                               int b_dtype, const void* q, const void* k, const void* v, void* o,
                               int qkv_dtype, const float* state, int64_t slot_stride,
                               const int32_t* chain, int chain_stride, const int32_t* depth,
                               const int32_t* init_slot, const int32_t* row_start,
                               const int32_t* row_count, int S, int n_max, float scale, int H,
                               int HV, int K, int V, void* stream);

/* cfb_tree_gdn without the states buffer, allocating nothing. This entry point has no
 * counterpart in the reference.
 * It is for callers that cannot allocate device memory when they verify: the verify step runs
 * inside the target model's forward pass, which serving engines record once into a CUDA graph
 * and replay, and no cudaMalloc may happen there; a caller that only needs o would otherwise
 * have to reserve a [B,N,H,Dk,Dv] fp32 states buffer for its largest batch up front.
 * The node states (which the kernel re-reads as parents) live in one fixed device array of
 * this library, CFB_TREE_GDN_NOALLOC_MAX_FLOATS fp32 (64 MiB), that every GPU which loads the
 * library holds until the process exits. Calls with B*N*H*Dk*Dv above that return
 * CFB_ERR_WORKSPACE. The first call on a device looks up the array's address on that device
 * (cudaGetSymbolAddress, with that device current): make that first call before any stream
 * capture. The address is kept for the life of the process, so a cudaDeviceReset of that device
 * after the first call is not supported (the kept address would be stale). Every call shares the array and leaves its node states there; none of it needs to
 * start at zero, but calls that overlap on the GPU (other streams, other host threads) race on
 * it, so order them on one stream. Arguments and supported shapes are those of cfb_tree_gdn. */
#define CFB_TREE_GDN_NOALLOC_MAX_FLOATS (16 * 1024 * 1024)
cfb_status cfb_tree_gdn_noalloc(const void* q, const void* k, const void* v, const float* g,
                                const float* beta, const int32_t* parent, const float* init,
                                float* o, int B, int N, int H, int Dk, int Dv, int use_l2norm,
                                void* stream);

/* ---- tree verification around the draft (the target model's side of a tree step) -------------
 * The tree-attention fix-up of one full-attention layer (the contract of the reference fork's
 * suffix_merge, src/chain_flow/patches/vllm-0.25.1-chain-flow-tree.patch:5516-5537, whose eager
 * form is _tree_suffix_eager :529-575 + vLLM's merge_attn_states): for request s and tree node m
 * (query row r = idx[s * N + m]) and query head h (key/value head h / (H / HKV)),
 *   suffix = softmax_n(scale * q[r, h] . k[idx[s, n], kh]) v[idx[s, n], kh] over the ancestors n
 *            of m (not_anc[(s * N + m) * N + n] == 0, m itself included), lse its log-sum-exp;
 *   o[r, h] = prefix_out[s * N + m, h] * ps / (ps + ss) + fp(suffix) * ss / (ps + ss),
 *            ps = exp(plse - M), ss = exp(lse - M), M = max(plse, lse), plse = prefix_lse[h, s*N + m]
 *            (a +inf lse counts as -inf), fp() = rounding to the I/O dtype.
 * q, k, v, o, prefix_out: fp16 (dtype 1) or bf16 (2) rows [*, heads, D] with the given strides in
 * elements (rows 16-byte aligned); prefix_lse fp32 [H, S * N]; idx int64 [S, N]; not_anc uint8
 * [S, N, N]. Only the tree rows of o are written. Supported: D in {64, 128, 256}, N <= 128,
 * H a multiple of HKV. */
cfb_status cfb_tree_attn_merge(const void* q, int64_t sq_t, int64_t sq_h, const void* k, int64_t sk_t,
                               int64_t sk_h, const void* v, int64_t sv_t, int64_t sv_h, void* o,
                               int64_t so_t, int64_t so_h, const void* prefix_out, int64_t spo_t,
                               int64_t spo_h, const float* prefix_lse, const int64_t* idx,
                               const uint8_t* not_anc, float scale, int S, int N, int H, int HKV,
                               int D, int dtype, void* stream);

/* Greedy tree verification (the contract of the reference fork's tree_rejection_sample and
 * tree_greedy_descent_kernel, src/chain_flow/patches/vllm-0.25.1-chain-flow-tree.patch:640-723):
 * the argmax of every logits row and the walk down each request's draft tree, in one launch.
 * Request r owns n = cu_num_draft[r] - cu_num_draft[r - 1] draft nodes (flat draft_tokens /
 * parents entries; parents are local node indices, -1 = the root) and logits rows [s0, s0 + n],
 * s0 = cu_num_sampled[r] - (n + 1): row s0 scores the committed token, row s0 + 1 + i node i.
 * From the root, the walk takes the row's argmax token (first maximum; NaN counts as the maximum,
 * as torch.argmax) and moves to the first child (node order) whose draft token equals it.
 * Outputs: output_tokens int32 [batch, max_spec_len + 1] = the accepted tokens then the bonus
 * token, -1 after; accepted_path int32 [batch, max_spec_len] = the accepted node indices, -1 after;
 * accepted_len int32 [batch]; row_argmax int32 [num_rows] (rows of the requests).
 * logits [num_rows, V] with row stride ld elements: fp32 (dtype 0), fp16 (1) or bf16 (2).
 * ws: cfb_tree_verify_workspace(num_rows, batch) bytes, 256-byte aligned, ZERO before its first
 * use (each launch leaves it zeroed again). err (may be NULL): set non-zero when a request's
 * offsets do not fit the logits rows or max_spec_len (that request then emits nothing).
 * Supported: max_spec_len <= 1024. */
size_t cfb_tree_verify_workspace(int num_rows, int batch);
cfb_status cfb_tree_verify_greedy(const void* logits, int64_t ld, int num_rows, int V, int dtype,
                                  const int32_t* cu_num_draft, const int32_t* cu_num_sampled,
                                  const int32_t* draft_tokens, const int32_t* parents, int batch,
                                  int max_spec_len, int32_t* output_tokens, int32_t* accepted_path,
                                  int32_t* accepted_len, int32_t* row_argmax, void* ws,
                                  size_t ws_bytes, int* err, void* stream);

/* ---- the per-request context ring -------------------------------------------------------------
 * The window of the last C target hidden states each request's draft is conditioned on
 * (reference FlowDrafterProposer._init_ring / _ring_write / _ring_gather,
 * flow_proposer.py:881-961). ring fp16 [slots, C + 1, H] (row C: trash row), rpos / nval int64
 * [slots] (next write position; valid rows <= C), all caller-owned, zero at start.
 * cfb_ring_write appends, for each of B requests (ring slot rows[b]), rows j < kmax taken from
 * the harvested hidden states sh fp16 [nsh, H]: sh[starts[b] + j] on a chain step (path NULL),
 * or sh[starts[b]] then sh[starts[b] + 1 + path[rows[b] * path_ld + j - 1]] on a tree step
 * (source rows clamped into sh); rows j >= cnt[b], and all rows of a request with wmask[b] == 0,
 * go to the trash row; rpos advances by cnt[b] mod C and nval saturates at C.
 * cfb_ring_gather writes out fp16 [B, C, H]: each slot's rows oldest first, front-padded by
 * repeating the oldest row when fewer than C exist. Both only move fp16 rows; the slots of one
 * call must be distinct. Supported: kmax <= 64 and C <= 64 (CFB_ERR_UNSUPPORTED beyond). */
cfb_status cfb_ring_write(void* ring, int64_t* rpos, int64_t* nval, int slots, int C, int H,
                          const void* sh, int64_t nsh, const int64_t* rows, const int64_t* starts,
                          const int64_t* cnt, const uint8_t* wmask, const int64_t* path,
                          int64_t path_ld, int B, int kmax, void* stream);
cfb_status cfb_ring_gather(const void* ring, const int64_t* rpos, const int64_t* nval, int slots,
                           int C, int H, const int64_t* rows, int B, void* out, void* stream);

/* ---- the wide (batched) drafting path ------------------------------------------------------
 * C = A · Wᵀ on the sm_100a tensor cores (tcgen05.mma, fp16 in, fp32 accumulate in TMEM), fed by
 * 2-D TMA copies: the GEMM of the wide path, exported on its own for tests and for callers that
 * batch their own rows. This entry point has no counterpart in the reference.
 * a fp16 [M, K] with row stride lda; w: an fp16 [N, ldw] matrix tiled by cfb_wide_pack (ldw a
 * multiple of 64, K <= ldw: the first K columns are multiplied); bias fp32 [N] or NULL.
 * epi: CFB_EPI_F32    out fp32 [M, ldo] = A·Wᵀ + bias
 *      CFB_EPI_F16    out fp16 [M, ldo] = fp16(A·Wᵀ + bias)
 *      CFB_EPI_GELU16 out fp16 [M, ldo] = fp16(gelu(A·Wᵀ + bias))   (exact erf GELU)
 *      CFB_EPI_PART   out fp32 [s][M, ldo]: split-K partials (bias ignored); s = ceil(K/64 /
 *                     ceil(K/64 / splits)) splits, each over a contiguous range of 64-column blocks.
 * Supported: K a multiple of 64, N a multiple of 16, a/w/out/bias 16-byte aligned, lda a
 * multiple of 8, ldo a multiple of 4. err: a device int that becomes non-zero if a bounded
 * device-side wait expired (outputs then invalid); it is never cleared by the library. */
enum { CFB_EPI_F32 = 0, CFB_EPI_F16 = 1, CFB_EPI_GELU16 = 2, CFB_EPI_PART = 3 };
/* The wide path's weight layout: an fp16 [nout, k] matrix (row stride ldw elements, k a multiple
 * of 64) as ceil(nout/256) x (k/64) blocks of 256 rows x 64 columns, block (n, j) at element
 * (n * k/64 + j) * 16384, each block the 128-byte-swizzled image the tensor cores read from shared
 * memory (16-byte chunk c of block row r stored at chunk c ^ (r mod 8)); rows past nout are zero.
 * One 32 KiB block per pipeline stage is one contiguous bulk copy. */
size_t cfb_wide_packed_bytes(int nout, int k);
cfb_status cfb_wide_pack(const void* w, int64_t ldw, int nout, int k, void* dst, void* stream);
cfb_status cfb_wide_gemm(const void* a, int64_t lda, const void* w, int64_t ldw, const float* bias,
                         void* out, int64_t ldo, int M, int N, int K, int epi, int splits, int* err,
                         void* stream);

/* The wide plan: a draft of many requests at once (the batch-throughput shape) as a fixed list
 * of kernel launches: tcgen05 GEMMs for every Linear (grouped over the chunk experts, split-K for
 * the residual projections), and row kernels for LayerNorm + residual updates, attention, the
 * path-token gather and the beam step. Same drafter description and run description as the
 * persistent plan, except that every cfb_linear.w is an fp16 [nout, k] matrix packed by
 * cfb_wide_pack, with the LayerNorm in front of it folded in (w = fp16(W * gamma),
 * bias = b + W beta); cfb_linear.colsum is unused. path_offsets is [D, order * D] (column block j
 * = offset_proj.j),
 * head is [R, Kh] = [lm_head[sl] | markov.w2[sl] | 0], Kh >= D + markov_rank a multiple of 64
 * (zero columns pad it). Modes and outputs are those of
 * cfb_run; the row-sharded head (ranks > 1) is not supported here. The library keeps the launch
 * list in host memory (cfb_wide_destroy frees it); all device memory is the caller's workspace.
 * cfb_wide_run only enqueues kernels on `stream` (capturable in a CUDA graph).
 * These entry points have no counterpart in the reference, whose batched drafts run its
 * per-layer PyTorch modules (reference cuda_block.py:382-431 for the fused expert). */
typedef struct cfb_wide_plan cfb_wide_plan;

/* The VAE bridge of the production drafter (reference TransformerHiddenVAE,
 * src/chain_flow/vae/transformer_hidden.py:51-67, as TreeVAEFlowDrafter._encode / _decode use
 * it, drafters/tree_vae_flow.py:163-175): one side (encoder or decoder) as a wide launch list.
 * in_proj [width, in_dim] (+ bias) then learned positions pos fp32 [max_len, width]; `layers`
 * pre-LN nn.TransformerEncoderLayer: qkv = self_attn.in_proj with norm1 folded in, attn_out =
 * self_attn.out_proj, ffn_up = linear1 with norm2 folded in (GELU), ffn_down = linear2; out_proj
 * with the side's final LayerNorm folded in (mu for the encoder, decoder_out for the decoder).
 * Every cfb_linear.w is packed by cfb_wide_pack (k = the packed inner dimension). */
typedef struct cfb_vae_layer { cfb_linear qkv, attn_out, ffn_up, ffn_down; } cfb_vae_layer;
typedef struct cfb_vae_side {
  int in_dim, width, out_dim, layers, heads, max_len;
  cfb_linear in_proj;
  const float* pos;
  const cfb_vae_layer* layer;
  cfb_linear out_proj;
} cfb_vae_side;
/* A plan of one side over `batch` requests of `rows` positions: encode (decode = 0) reads
 * fp16 [batch, rows, in_dim] and writes fp16 [batch, rows, out_dim] (mu, the flow's context);
 * decode (decode = 1) reads fp32 [batch, rows, in_dim] (the integrated latent) and writes fp32
 * [batch, rows, out_dim] (the hidden states the head scores). The plan is run, checked and freed
 * with cfb_wide_run / cfb_wide_error / cfb_wide_destroy. Supported: in_dim and width multiples of
 * 64, out_dim a multiple of 16, width / heads a multiple of 8, rows <= 16 and <= max_len. */
cfb_status cfb_vae_workspace(const cfb_vae_side* v, int batch, int rows, int decode, size_t* bytes);
/* The same side as a persistent-engine plan (batch * rows <= 64: the small batches, where one
 * cooperative launch beats a launch list): every cfb_linear packed by cfb_pack_linear, the
 * LayerNorms folded by cfb_fold_bias (colsum set for qkv, ffn_up and out_proj). I/O as for
 * cfb_vae_create; the plan lives in the caller's workspace and runs with cfb_plan_run /
 * cfb_plan_error like a drafting plan. */
cfb_status cfb_vae_plan_workspace(const cfb_vae_side* v, int batch, int rows, int decode, size_t* bytes);
cfb_status cfb_vae_plan_build(const cfb_vae_side* v, int batch, int rows, int decode, const void* in,
                              void* out, void* ws, size_t bytes);
cfb_status cfb_vae_create(const cfb_vae_side* v, int batch, int rows, int decode, const void* in,
                          void* out, void* ws, size_t bytes, cfb_wide_plan** plan);
cfb_status cfb_wide_workspace(const cfb_drafter* d, const cfb_run* r, size_t* bytes);
cfb_status cfb_wide_create(const cfb_drafter* d, const cfb_run* r, void* ws, size_t bytes,
                           cfb_wide_plan** plan);
cfb_status cfb_wide_run(cfb_wide_plan* plan, void* stream);
/* synchronous read of the sticky device error word (0 = every run so far completed) */
cfb_status cfb_wide_error(cfb_wide_plan* plan, int* device_error);
cfb_status cfb_wide_info(cfb_wide_plan* plan, int* launches);
void cfb_wide_destroy(cfb_wide_plan* plan);

#ifdef __cplusplus
}
#endif
#endif /* CFB_H_ */
