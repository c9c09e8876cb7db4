/*
 * rtr_b200.h - C ABI of the B200-native semantic-ID beam-search engine.
 *
 * One session = one model replica on one GPU serving sequential requests
 * (batch 1, 50 beams, 3 SID tokens + newline + EOS), which is how the
 * reference runs (rapidtinyrec/benchmark_inference.py:62-258; one model, one
 * stream, one isolated worker: docs/release-scope.md:41-44).
 *
 * Conventions
 *   - Every entry point returns an int status: RTR_OK (0) or an RTR_ERR_*
 *     code.  No exception crosses the ABI.  rtr_last_error() gives the text.
 *   - RTR_ERR_ARG mirrors the reference's ValueError (shape, capacity,
 *     aliasing: shared_prefix.py:71-73, prefix_replay.py:99-101);
 *     RTR_ERR_STATE its RuntimeError (call order, frozen pools:
 *     decode_replay.py:185, inference_precision.py:53-54).
 *   - Pointers are plain host or device addresses; sizes are element counts.
 *     "dev" parameters must be device memory of the session's GPU; "host"
 *     parameters are host memory (pinned memory makes the copies async).
 *   - The caller owns every buffer it passes; the session owns its device
 *     state (weights, constraint tables, prefix arena, beam state).
 *   - A session is not thread-safe; use one session per GPU per process.
 *     All device work is issued on the session's stream (rtr_set_stream).
 */
#ifndef RTR_B200_H
#define RTR_B200_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define RTR_OK 0
#define RTR_ERR_ARG 1     /* invalid argument, shape or capacity          */
#define RTR_ERR_STATE 2   /* wrong call order / missing weights or tables */
#define RTR_ERR_CUDA 3    /* CUDA runtime error                           */
#define RTR_ERR_DEVICE 4  /* a device-side check failed (see message)     */

#define RTR_DTYPE_F32 0
#define RTR_DTYPE_BF16 1

#define RTR_NUM_STEPS 5   /* prefill output + 4 decode forwards */

typedef struct rtr_session rtr_session;

/* Model shape.  Mirrors the Qwen2 config fields the reference reads from the
 * release (benchmark_inference.py:93-98) plus the runtime capacities of the
 * prefix arena (shared_prefix.py:53-65). */
typedef struct {
  int32_t layers, hidden, heads, kv_heads, head_dim, intermediate, vocab;
  int32_t tied_embeddings;  /* lm_head shares the embedding matrix */
  float rms_eps;
  float rope_theta;
  int32_t dtype;            /* RTR_DTYPE_F32 / RTR_DTYPE_BF16: weights, activations, KV */
  int32_t max_prefix;       /* prefix arena capacity in tokens (PrefixArena max_prefix_tokens) */
  int32_t num_beams;        /* 50 in the reference (benchmark_inference.py:139) */
} rtr_model_config;

/* Dense SID constraint tables, int32 copies of GpuSidConstraintTables
 * (gpu_constraints.py:31-60): offsets/sizes of the three SID levels, the
 * step-1 table [sizes[0] x width1], the step-2 table
 * [sizes[0]*sizes[1] x width2] (rows padded by repeating their first token),
 * the validity bitmap over sizes[0]*sizes[1]*sizes[2] (one byte each), the
 * root prefix and the sorted first tokens.  All pointers are host memory. */
typedef struct {
  int32_t offsets[3], sizes[3];
  const int32_t* table1; int32_t width1;
  const int32_t* table2; int32_t width2;
  const uint8_t* valid;
  int32_t root[3];
  const int32_t* first_tokens; int32_t n_first;
  int32_t newline, eos;
} rtr_constraint_tables;

/* Per-request result, host buffers sized by num_beams B (the reference's
 * per-user record, benchmark_inference.py:150-154 / 241-244):
 *   token_ids[B*5]       generated tokens of the ranked beams (int32)
 *   beam_indices[B*5]    parent beam row at every step
 *   sequence_logp[B]     FP32 sequence scores (sequences_scores)
 *   transition_logp[B*5] FP32 per-step scores (compute_transition_scores)  */
typedef struct {
  int32_t* token_ids;
  int32_t* beam_indices;
  float* sequence_logp;
  float* transition_logp;
} rtr_result;

/* ---- session lifecycle -------------------------------------------------- */

/* Replaces the model/compiler/arena/pool set-up of
 * benchmark_inference.py:93-121 (CompiledForward, PrefixArena,
 * PrefixReplayPool, ReorderSuffix).  Allocates all device state. */
int rtr_session_create(const rtr_model_config* cfg, int device, rtr_session** out);
/* The same session sized for up to max_users (1..8) users per request: each
 * user gets its own prefix arena, beam state and result; rtr_launch_batch runs
 * their decode steps together (no reference counterpart: the reference serves
 * one user per request). */
int rtr_session_create_batched(const rtr_model_config* cfg, int device, int32_t max_users, rtr_session** out);
int rtr_session_destroy(rtr_session* s);

/* Text of the last error of this session (or of the last failed create when
 * s is NULL).  Valid until the next call on the session. */
const char* rtr_last_error(const rtr_session* s);

/* Issue all work of the session on this cudaStream_t (NULL = session-owned
 * stream).  Invalidates captured graphs. */
int rtr_set_stream(rtr_session* s, void* stream);

/* Load weights in the canonical Qwen2 order: embed [V,H]; per layer
 * q_w [Hq*D,H], q_b, k_w [Hkv*D,H], k_b, v_w, v_b, o_w [H,Hq*D],
 * gate_w [I,H], up_w [I,H], down_w [H,I], input_norm [H], post_norm [H];
 * final_norm [H]; lm_head [V,H] unless tied.  n_tensors = 1 + 12*layers + 1
 * (+1 untied).  src_dtype is the element type of the given tensors
 * (converted with round-to-nearest-even when it differs from the session
 * dtype); src_on_device selects device or host pointers.
 * Replaces from_pretrained(...).to('cuda') (benchmark_inference.py:93-98). */
int rtr_load_weights(rtr_session* s, const void* const* tensors, int32_t n_tensors,
                     int32_t src_dtype, int32_t src_on_device);

/* RoPE cos/sin tables [n_positions, head_dim/2] float32, host memory
 * (Qwen2RotaryEmbedding, transformers modeling_qwen2.py:89-113).  Optional:
 * without it the session computes them on the host in double precision. */
int rtr_load_rope(rtr_session* s, const float* cos_host, const float* sin_host, int32_t n_positions);

/* Upload the constraint tables.  Replaces GpuSidConstraintTables(...,
 * device='cuda') (gpu_constraints.py:18-67, benchmark_inference.py:92). */
int rtr_load_constraints(rtr_session* s, const rtr_constraint_tables* t);

/* ---- one request ---------------------------------------------------------- */

/* Prefill one request of L tokens into the single shared prefix copy and run
 * step 0 (normalisation, mask, beam top-k).  ids may be host or device
 * (ids_on_device).  Replaces PrefillPrefix.forward + PrefixArena.start_request
 * + the first _beam_search iteration (prefix_prefill.py:27-63,
 * shared_prefix.py:67-89). */
int rtr_prefill(rtr_session* s, const int32_t* ids, int32_t L, int32_t ids_on_device);

/* Decode step t in 1..4: 50-row forward over the shared prefix and the beams'
 * suffixes, full-vocabulary double log-softmax, trie mask, beam top-k and the
 * suffix parent gather, all on device without a host round trip.  Replaces
 * one _beam_search iteration with PrefixReplayPool.__call__,
 * GpuSidConstrainedLogitsProcessor.__call__ and ReorderSuffix.reorder
 * (decode_replay.py:180-191, gpu_constraints.py:95-101,
 * prefix_replay.py:95-117). */
int rtr_decode_step(rtr_session* s, int32_t t);

/* Copy the finished ranking to host buffers (blocking on the stream).  Fails
 * with RTR_ERR_DEVICE when the beam loop would not have stopped after five
 * steps or a device-side bound check fired.  Replaces unpack
 * (benchmark_inference.py:150-154). */
int rtr_read_results(rtr_session* s, const rtr_result* out);

/* Whole request: prefill + steps 1..4 (one CUDA graph) + result copy.
 * Replaces benchmark_inference.generate (:123-148). */
int rtr_generate(rtr_session* s, const int32_t* ids_host, int32_t L, const rtr_result* out);

/* Batched requests (sessions from rtr_session_create_batched): n_users prompts
 * ids[u] of lengths L[u]; every user's prefill runs on its own, then one decode
 * graph runs steps 1-4 for all n users, each projection GEMM at n x beams rows.
 * Each user's ranking equals its batch-1 result (same kernels and, up to two
 * users, the same split-K partition; beyond that the GEMM partition can change
 * the last bits).  out points to n_users results.  One status word covers the
 * batch: a device check that fails for one user fails the batch. */
int rtr_launch_batch(rtr_session* s, const int32_t* const* ids, const int32_t* L, int32_t n_users,
                     int32_t ids_on_device);
int rtr_wait_batch(rtr_session* s, const rtr_result* out);
int rtr_generate_batch(rtr_session* s, const int32_t* const* ids_host, const int32_t* L, int32_t n_users,
                       const rtr_result* out);

/* The two halves of rtr_generate for callers that overlap requests with host
 * work: rtr_launch enqueues prefill + the decode graph + the result copy on the
 * session stream and returns without waiting (ids host or device);
 * rtr_wait blocks until the last launched request finished, checks it and
 * fills out (NULL out: check only).  Requests with device ids may be queued
 * back to back (the stream orders them; only the last one's result is kept);
 * a launch with host ids first waits for the request in flight, because the
 * prompt is staged through one pinned buffer. */
int rtr_launch(rtr_session* s, const int32_t* ids, int32_t L, int32_t ids_on_device);
int rtr_wait(rtr_session* s, const rtr_result* out);

/* Counters of the session, the counterpart of the reference's report()
 * records (PrefixReplayPool.report, PrefixArena.report, ReorderSuffix.report:
 * decode_replay.py:193-202, shared_prefix.py:110-116, prefix_replay.py:242-244). */
typedef struct {
  int64_t requests;               /* requests launched                         */
  int64_t kernel_launches;        /* kernels issued, graph nodes included      */
  int64_t launches_per_request;   /* kernels one request issues                */
  int64_t graph_kernel_nodes;     /* kernel nodes of the decode graph          */
  int64_t prefix_bytes_written;   /* prefix K/V written by the last prefill    */
  int64_t prefix_bytes_reordered; /* always 0: the prefix is shared in place   */
  int64_t suffix_bytes_written;   /* suffix K/V written per request            */
  int64_t suffix_bytes_gathered;  /* 0: parents are followed through anc rows  */
  int64_t weight_bytes;           /* resident weight bytes                     */
  int64_t device_bytes;           /* all device memory the session holds       */
  int64_t h2d_bytes_per_request;  /* prompt ids + length                       */
  int64_t d2h_bytes_per_request;  /* the result record                         */
  int64_t tensor_core_gemm;       /* 2: tcgen05 fp16-pair projections (fp32
                                     default), 1: tcgen05 3xTF32, 0: FFMA      */
  int64_t norm_fold;              /* 1: RMSNorms folded into the GEMMs         */
  int64_t decode_attention;       /* 0: per-head kernel (fp32 default,
                                     RTR_ATTN=rows), 1: tensor-core folded
                                     kernel (bf16 default, fp32 RTR_ATTN=tc),
                                     2: folded FFMA kernel (RTR_ATTN=folded)   */
  int64_t prefill_attention;      /* 0: FFMA kernel, 1: tensor-core kernel
                                     (default; RTR_PREFILL_ATTN=ffma)          */
} rtr_report;
int rtr_get_report(const rtr_session* s, rtr_report* out);

/* Measurement hook (no reference counterpart): run every projection GEMM of
 * one forward pass over M rows (q/k/v, o, gate/up, down per layer, then the
 * LM head) `reps` times on the session stream and return the average device
 * milliseconds of one pass, timed with CUDA events.  Activations are
 * scratch; the session must not have a request in flight. */
int rtr_profile_gemms(rtr_session* s, int32_t M, int32_t reps, float* ms_per_pass);

/* Test hook (no reference counterpart): C[M, N] = X[M, K] . W[N, K]^T (fp32,
 * row-major, device pointers) through one projection-GEMM kernel: 0 the
 * engine's fp32 dispatch (= 5), 1 the 64-row tcgen05 3xTF32 kernel, 2 the
 * 128-row one, 3 the bf16 kernel (X and W rounded to bf16 first; C holds the
 * bf16-rounded products as fp32), 4 the FFMA kernel, 5 the tcgen05 fp16-pair
 * kernel (X and W as fp16 (hi, lo) pairs; 64-row CTAs for M <= 64, else
 * 128-row).  N must be a multiple of 4 and K of 4 (8 for the bf16 and
 * fp16-pair kernels, 32 for FFMA).  Scratch is allocated per call; blocks
 * until done. */
int rtr_gemm_check(int32_t device, const float* x_dev, const float* w_dev, float* c_dev, int32_t M, int32_t N,
                   int32_t K, int32_t kernel);

/* Test hook (no reference counterpart): causal prefill attention of one layer
 * of one user, out[L, heads, D] = softmax(q k^T / sqrt(D), causal) v with the
 * query heads of KV group g = h / (heads / kv_heads) reading k, v [g] (fp32,
 * row-major, device pointers; k and v [kv_heads, L, D]) through one kernel:
 * 0 the FFMA kernel, 1 the tensor-core fp16-pair kernel, 2 the bf16 FFMA
 * kernel and 3 the bf16 tensor-core kernel (2 and 3: q, k, v rounded to bf16
 * first, out holds the bf16 results).  head_dim 64 or 128.  Builds the arena
 * and copies the kernel reads; scratch is allocated per call; blocks until
 * done. */
int rtr_attention_check(int32_t device, const float* q_dev, const float* k_dev, const float* v_dev, float* out_dev,
                        int32_t L, int32_t heads, int32_t kv_heads, int32_t head_dim, int32_t kernel);

/* Test hook (no reference counterpart; the reference's failure handling is
 * Python exceptions): on `device`, bound every pipeline wait of the
 * fp16-pair and bf16 tensor-core GEMMs to wait_cycles (default 2e9, ~1 s) and,
 * with withhold_activation_copies = 1, make their activation producers issue
 * no copy.  Those waits then run out: each CTA stops issuing, drains what it
 * issued, frees its tensor memory, keeps the split-K tickets whole and sets the
 * timeout bit of the session's status word, so the request fails with
 * RTR_ERR_DEVICE and the next request runs normally.  Applies to kernels
 * launched (or graph nodes replayed) after the call; wait_cycles >= 1000.
 * Blocks until the setting is on the device. */
int rtr_debug_wait_control(int32_t device, int64_t wait_cycles, int32_t withhold_activation_copies);

/* Processed scores of step t (0..4) as a dense [B, V] float32 device matrix:
 * the double-normalised log-probabilities at allowed columns and -inf
 * elsewhere, i.e. GenerateBeamOutput.scores[t] (the --save-full-scores
 * payload, benchmark_inference.py:160-172). */
int rtr_step_scores(rtr_session* s, int32_t t, float* out_dev);

/* ---- plugin-level entry points (the reference's LogitsProcessor API) ---- */

/* GpuSidConstraintTables.lookup (gpu_constraints.py:75-87): allowed columns
 * for input_ids [rows, cols] (int64, device) at step; out_dev [rows, width]
 * int32 where width = n_first at steps 0/3, width1 / width2 at steps 1/2 and 1
 * afterwards (rtr_lookup_width). */
int rtr_lookup_width(const rtr_session* s, int32_t step, int32_t* width);
int rtr_constraint_lookup(rtr_session* s, int32_t step, const int64_t* input_ids_dev,
                          int32_t rows, int32_t cols, int32_t* out_dev);

/* GpuSidConstrainedLogitsProcessor.__call__ (gpu_constraints.py:95-101):
 * out = log_softmax(scores) + mask(lookup(step, input_ids)); scores and out
 * are [rows, V] float32 device matrices (out may not alias scores). */
int rtr_constraint_process(rtr_session* s, int32_t step, const int64_t* input_ids_dev,
                           int32_t rows, int32_t cols, const float* scores_dev, float* out_dev);

/* Allocation-free rtr_constraint_process.  No counterpart in the reference.
 * For callers that must not allocate device memory per call - a plugin whose
 * host framework owns the GPU allocator and has reserved the memory, or a
 * serving loop whose latency budget rules out the allocator's synchronisation.
 * It computes the same scores with the same kernels, but keeps the per-row
 * reduction scratch in a fixed static device array of the library instead of
 * session memory, and it calls no cudaMalloc, cudaFree or allocating routine.
 * Limits and caveats:
 *   - rows <= 256 (the array's size: 256 rows x 16 slices x 2 floats = 32 KiB,
 *     held by every GPU that loads the library until the process exits);
 *     larger requests fail with RTR_ERR_ARG;
 *   - the first call on a device looks the array's device address up once
 *     (cudaGetSymbolAddress) and keeps it; do not call cudaDeviceReset on
 *     that device afterwards (the kept address would be stale);
 *   - all calls share the one array, so calls whose work overlaps on the GPU
 *     (other streams, other sessions on the same device) race on it; nothing
 *     needs clearing between calls, because each call writes every slot it
 *     reads before reading it;
 *   - blocks until the scores are written. */
int rtr_constraint_process_static(rtr_session* s, int32_t step, const int64_t* input_ids_dev,
                                  int32_t rows, int32_t cols, const float* scores_dev, float* out_dev);

/* ---- synthetic workload --------------------------------------------------- */

/* Deterministic synthetic tensor values: element i of stream (seed, tid) is
 * (k - 2^23) * (scale * 2^-23) + offset, k = top 24 bits of
 * splitmix64(key(seed, tid) + i * golden).  Host (multi-threaded) and device
 * fills are bit-identical.  No reference counterpart: it generates the
 * stand-in for the unavailable release checkpoint. */
int rtr_synth_fill_host(float* dst, int64_t n, uint64_t seed, uint64_t tid, float scale, float offset);
int rtr_synth_fill_device(float* dst_dev, int64_t n, uint64_t seed, uint64_t tid, float scale,
                          float offset, void* stream);

#ifdef __cplusplus
}
#endif
#endif /* RTR_B200_H */
