// Internal declarations shared by the engine's translation units.
#pragma once

#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

namespace rtr {

enum Epilogue : int { EPI_STORE = 0, EPI_BIAS = 1, EPI_RESID = 2, EPI_SWIGLU = 3, EPI_ROPE = 4 };

// EPI_ROPE (tensor-core GEMM only): the q/k/v projection's epilogue adds the
// bias, applies RoPE to q and k and writes q to q_out [M][heads*D] and k/v to
// the cache, exactly as rope_kv() below does from a stored projection.
struct RopeArgs {
  const float* cos_t;
  const float* sin_t;
  int positions;           // rows of the cos/sin tables
  int heads, kv_heads, head_dim;
  float* q_out;
  float* k_dst;
  float* v_dst;
  int prefix_cap;
  int slot;                // < 0: prefill (row m at position m); else decode suffix slot
  const int32_t* L_dev;    // decode: prefix length (position = *L_dev + slot)
  int rows_per_user = 0;   // batched decode: row m belongs to user m / rows_per_user (L_dev[user])
  // prefill only, when set: the prefix K and V also as fp16 pairs for the
  // tensor-core decode attention (the layer's group-0 bases): K as
  // [group][pair_cap][head_dim] hi / lo planes, V transposed as
  // [group][head_dim][pair_cap] hi / lo planes
  void* kpair_hi = nullptr;
  void* kpair_lo = nullptr;
  void* vtpair_hi = nullptr;
  void* vtpair_lo = nullptr;
  int pair_cap = 0;
};

// RMSNorm folded into the projection GEMMs (fp32 tensor-core paths): the norm
// weight is folded into the packed weight's columns, the producer of the
// residual stream (embedding, o_proj / down_proj epilogues) writes x's split
// (SPLIT_F16 pair or SPLIT_TF32) and per-row
// partial sums of squares over 128-column chunks (ss[chunk * ld + row]), and
// the consuming GEMM scales each output row by 1 / sqrt(sum / hidden + eps).
struct NormFold {
  float* ss_out;           // producer (EPI_RESID): partial sums of squares of the new x
  const float* ss_in;      // consumer: partials of the GEMM's input rows
  int ld;                  // row stride of a chunk's partials (rows capacity)
  int parts;               // chunks per row (hidden / 128)
  int hidden;
  float eps;
};

// ---- GEMM (gemm_ffma.cu) ----
cudaError_t gemm_init();
size_t gemm_workspace_floats(int max_m, int max_n, int sms);
int gemm_tile_count(int max_m, int max_n);
cudaError_t gemm_f32(const float* A, int lda, const float* W, float* C, int ldc, const float* bias,
                     int M, int N, int K, int epi, float* ws, size_t ws_floats, int* tickets,
                     int sms, cudaStream_t stream, bool pdl);
cudaError_t gemv_f32(const float* x, const float* W, float* y, int N, int K, cudaStream_t stream);

// ---- tensor-core GEMM (gemm_tc.cu): 3xTF32 on tcgen05 ----
struct alignas(64) TensorMap { unsigned char bytes[128]; };  // a CUtensorMap
// fp32 row-major [rows][cols], row stride ld floats; TMA box [box_rows][32]
bool make_tmap_f32(TensorMap* out, const float* base, long rows, long cols, long ld, int box_rows);
cudaError_t gemm_tc_init();
// Weights are packed once into tile-contiguous blocks for the tensor-core GEMM.
size_t packed_weight_floats(int N, int K);
cudaError_t pack_weight_tiles(const float* src, int N, int K, float* dst, cudaStream_t stream,
                              const float* col_scale = nullptr);  // W[n][k] * col_scale[k] when given
bool make_tmap_packed(TensorMap* out, const float* packed, int N, int K);
// Activations are consumed as a (big, small) pair: big = tf32(x), small = x - big.
cudaError_t gemm_tc(const TensorMap& tmW, const TensorMap& tmXb, const TensorMap& tmXs, float* C, float* C_big,
                    float* C_small, int ldc, const float* bias, int M, int N, int K, int epi, float* ws,
                    size_t ws_floats, int* tickets, int max_tickets, uint32_t* status, int sms, cudaStream_t stream,
                    bool pdl, const RopeArgs* rope = nullptr, const NormFold* fold = nullptr);
// The same GEMM with 128 activation rows per CTA (gemm_tc_wide.cu): for M > 64.
cudaError_t gemm_tc_wide_init();
cudaError_t gemm_tc_wide(const TensorMap& tmW, const TensorMap& tmXb, const TensorMap& tmXs, float* C, float* C_big,
                         float* C_small, int ldc, const float* bias, int M, int N, int K, int epi, float* ws,
                         size_t ws_floats, int* tickets, int max_tickets, uint32_t* status, int sms,
                         cudaStream_t stream, bool pdl, const RopeArgs* rope = nullptr,
                         const NormFold* fold = nullptr);

// ---- fp16-pair tensor-core GEMM (gemm_f16x2.cu): the fp32 path's default ----
// Weights packed once as fp16 (hi, lo) pairs (4 bytes a weight); activations
// consumed as SPLIT_F16 planes (hi, lo) written by their producers.  Same
// arguments, epilogues and split-K as gemm_tc; 64-row CTAs for M <= 64,
// 128-row CTAs above.
size_t packed_weight_elems_f16x2(int N, int K);
cudaError_t pack_weight_tiles_f16x2(const float* src, int N, int K, void* dst, cudaStream_t stream,
                                    const float* col_scale = nullptr);
// fp16 row-major [rows][cols], row stride ld elements; TMA box [box_rows][64]
bool make_tmap_f16(TensorMap* out, const void* base, long rows, long cols, long ld, int box_rows);
bool make_tmap_packed_f16x2(TensorMap* out, const void* packed, int N, int K);
cudaError_t gemm_f16x2_init();
// Test control of the fp16-pair and bf16 GEMMs on the current device: the
// bound of their pipeline waits (cycles) and a switch that makes their
// activation producers issue no copy (so those waits run out).
cudaError_t gemm_f16x2_wait_control(long long wait_cycles, int withhold_x);
cudaError_t gemm_bf16_wait_control(long long wait_cycles, int withhold_x);
cudaError_t gemm_f16x2(const TensorMap& tmW, const TensorMap& tmXh, const TensorMap& tmXl, float* C, float* C_big,
                       float* C_small, int ldc, const float* bias, int M, int N, int K, int epi, float* ws,
                       size_t ws_floats, int* tickets, int max_tickets, uint32_t* status, int sms, cudaStream_t stream,
                       bool pdl, const RopeArgs* rope = nullptr, const NormFold* fold = nullptr, float2* lse = nullptr, int lse_ld = 0);

// ---- bf16 tensor-core GEMM (gemm_bf16.cu): the bf16 mode ----
// X: bf16 activations [rows][K]; weights packed once into bf16 tile blocks.
// C is bf16 except EPI_STORE (fp32 copies of the bf16 logits); bias holds bf16
// values in fp32; EPI_ROPE writes bf16 q and cache rows.
bool make_tmap_bf16(TensorMap* out, const void* base, long rows, long cols, long ld, int box_rows);
cudaError_t gemm_bf16_init();
size_t packed_weight_elems_bf16(int N, int K);
cudaError_t pack_weight_tiles_bf16(const float* src, int N, int K, void* dst, cudaStream_t stream);
bool make_tmap_packed_bf16(TensorMap* out, const void* packed, int N, int K);
cudaError_t gemm_bf16(const TensorMap& tmW, const TensorMap& tmX, void* C, int ldc, const float* bias, int M, int N,
                      int K, int epi, float* ws, size_t ws_floats, int* tickets, int max_tickets, uint32_t* status,
                      int sms, cudaStream_t stream, bool pdl, const RopeArgs* rope = nullptr,
                      float2* lse = nullptr, int lse_ld = 0, bool allow_wide = true);

// ---- element-wise (elementwise.cu) ----
// x = table[ids]; with x_big/x_small (optional) also x's GEMM split (format
// xfmt: SPLIT_TF32 or SPLIT_F16, common.cuh) and, with ss (optional), x's
// per-row partial sums of squares (NormFold layout).
cudaError_t embed_rows(const int32_t* ids, int ids_stride, int M, const float* table, int vocab,
                       int hidden, float* x, uint32_t* status, cudaStream_t stream, float* x_big = nullptr,
                       float* x_small = nullptr, float* ss = nullptr, int ss_ld = 0, int grp_rows = 0,
                       long grp_stride = 0,  // row m: ids[(m / grp_rows) * grp_stride + (m % grp_rows) * ids_stride]
                       int xfmt = 0);
// h = w * (x * rsqrt(mean(x^2) + eps)); h_big/h_small (optional) get the GEMM split of h.
cudaError_t rms_norm_rows(const float* x, const float* w, float* h, float* h_big, float* h_small, int M, int hidden,
                          float eps, cudaStream_t stream, int xfmt = 0);
// RoPE on q and k of a [M, qkv_dim] projection; q -> q_out [M, Hq*D], k/v ->
// cache rows.  Prefill (slot < 0): row m is position m, K/V go to the prefix
// arena [Hkv][cap][D] at position m.  Decode (slot >= 0): every row is at
// position *L_dev + slot, K/V go to suffix slot `slot` [beams][Hkv][D].
cudaError_t rope_kv(const float* qkv, int M, int heads, int kv_heads, int head_dim,
                    const float* cos_t, const float* sin_t, int rope_positions,
                    float* q_out, float* k_dst, float* v_dst, int prefix_cap,
                    int slot, const int32_t* L_dev, uint32_t* status, cudaStream_t stream);
cudaError_t synth_fill_device(float* dst, int64_t n, uint64_t seed, uint64_t tid, float scale,
                              float offset, cudaStream_t stream);
void synth_fill_host(float* dst, int64_t n, uint64_t seed, uint64_t tid, float scale, float offset);
cudaError_t f32_to_bf16(const float* src, void* dst, int64_t n, cudaStream_t stream);
// bf16 mode (bf16 activations; norm weights and biases as bf16 values in fp32)
cudaError_t embed_rows_bf16(const int32_t* ids, int ids_stride, int M, const void* table, int vocab, int hidden,
                            void* x, uint32_t* status, cudaStream_t stream, int grp_rows = 0, long grp_stride = 0);
cudaError_t rms_norm_rows_bf16(const void* x, const float* w, void* h, int M, int hidden, float eps,
                               cudaStream_t stream);
cudaError_t gemv_bf16(const void* x, const void* W, float* y, int N, int K, cudaStream_t stream);
cudaError_t round_to_bf16(float* v, int64_t n, cudaStream_t stream);

// ---- attention (attention.cu) ----
// out_big/out_small (optional, fp32 only) receive the GEMM split of out
// (format xfmt).  bf16: q, K/V and out are bf16 (the bf16 mode); otherwise fp32.
cudaError_t attention_prefill(const void* q, const void* k_prefix, const void* v_prefix, void* out, float* out_big,
                              float* out_small, int L, int prefix_cap, int heads, int kv_heads, int head_dim,
                              float scale, bool bf16, cudaStream_t stream, int xfmt = 0);
// Users of a batched decode step: user u owns rows u * beams .. u * beams + beams - 1,
// its prefix at k/v_prefix + u * prefix_user_stride, its length L_dev[u] and its
// ancestry table at anc + u * anc_user_stride.
struct DecodeUsers {
  int users = 1;
  long prefix_user_stride = 0;  // elements
  int anc_user_stride = 0;      // int32 elements
};
// Decode attention over the shared prefix (length L_dev[user]) and `t` suffix
// slots; suffix slot s of beam b lives in row anc[b*4+s] (slot t-1: row b).
cudaError_t attention_decode(const void* q, const void* k_prefix, const void* v_prefix, const void* k_suffix,
                             const void* v_suffix, const int32_t* anc, const int32_t* L_dev, int t, void* out,
                             float* out_big, float* out_small, int beams, int prefix_cap, int heads, int kv_heads,
                             int head_dim, float scale, uint32_t* status, bool bf16, cudaStream_t stream,
                             const DecodeUsers& du = DecodeUsers{}, int xfmt = 0);
cudaError_t attention_init();
// Folded decode attention (attn_decode.cu): the rows of KV group g are its
// (beam, head) pairs; a cluster of 8 CTAs splits the prefix keys, staged by
// TMA through `arena`, a 2-D map over the prefix arena with rows of head_dim
// elements, boxes of 32 rows x 128 bytes, 128-byte swizzle.  krow0 / vrow0:
// the arena rows of the layer's K / V of group 0 of user 0; user_rows: arena
// rows per user.  Same arguments and results as attention_decode otherwise.
cudaError_t attention_decode_folded(const TensorMap& arena, long krow0, long vrow0, long user_rows, const void* q,
                                    const void* k_suffix, const void* v_suffix, const int32_t* anc,
                                    const int32_t* L_dev, int t, void* out, float* out_big, float* out_small,
                                    int beams, int prefix_cap, int heads, int kv_heads, int head_dim, float scale,
                                    uint32_t* status, bool bf16, cudaStream_t stream, const DecodeUsers& du,
                                    int xfmt);
cudaError_t attention_folded_init();

// Tensor-core decode attention (attn_tc.cu): the prefix K and V as fp16 pairs
// (written by the prefill's q/k/v epilogue), K [row][head_dim] and V
// transposed [row][pair_cap], each with a hi plane and, `*plane` rows
// further, a lo plane.  krow0 / vrow0: the rows of the layer's group 0 of user
// 0; kuser / vuser: rows per user; groups are pair_cap (K) or head_dim (V)
// rows apart.  Prompts of up to 448 tokens, fp32 mode.
struct AttnPairs {
  TensorMap kmap, vmap;
  long krow0, kplane, kuser, vrow0, vplane, vuser;
  int pair_cap;
};
bool attention_tc_supported(int heads, int kv_heads, int head_dim, int max_prefix);
cudaError_t attention_decode_tc(const AttnPairs& ap, const float* q, const float* k_suffix, const float* v_suffix,
                                const int32_t* anc, const int32_t* L_dev, int t, float* out, float* out_big,
                                float* out_small, int beams, int prefix_cap, int heads, int kv_heads, int head_dim,
                                float scale, uint32_t* status, cudaStream_t stream, const DecodeUsers& du, int xfmt);
cudaError_t attention_tc_init();
// Causal prefill attention of user `user`'s prompt (L tokens) on the tensor
// cores, from the pair copies the layer's q/k/v epilogue wrote (ap.krow0 /
// ap.vrow0 set to the layer, as for attention_decode_tc); fp32 mode.
bool attention_prefill_tc_supported(int heads, int kv_heads, int head_dim);
cudaError_t attention_prefill_tc(const AttnPairs& ap, int user, const float* q, float* out, float* out_big,
                                 float* out_small, int L, int heads, int kv_heads, int head_dim, float scale,
                                 uint32_t* status, cudaStream_t stream, int xfmt);
// The bf16 mode's tensor-core prefill attention: K by TMA from the bf16 prefix
// arena (kmap: the arena as [rows][head_dim], 64-row boxes), V from the
// transposed copy the bf16 q/k/v epilogue writes ([user][layer][group][dim]
// [pair_cap], vmap: head_dim-row boxes).
struct BfPrefillMaps {
  TensorMap kmap, vmap;
  int pair_cap;
};
cudaError_t attention_prefill_tc_bf16(const BfPrefillMaps& mp, int user, int layer, int layers, const void* q,
                                      void* out, int L, int heads, int kv_heads, int head_dim, int cap, float scale,
                                      uint32_t* status, cudaStream_t stream);
// The bf16 mode's decode attention on the tensor cores (any prefix the arena
// holds; the same arena map and V copy as the prefill kernel).
bool attention_decode_tc_bf16_supported(int heads, int kv_heads, int head_dim);
cudaError_t attention_decode_tc_bf16(const BfPrefillMaps& mp, int layer, int layers, const void* q,
                                     const void* k_suffix, const void* v_suffix, const int32_t* anc,
                                     const int32_t* L_dev, int t, void* out, int beams, int prefix_cap, int heads,
                                     int kv_heads, int head_dim, float scale, uint32_t* status, cudaStream_t stream,
                                     const DecodeUsers& du);
bool attention_folded_supported(int heads, int kv_heads, int head_dim, bool bf16);

// ---- constraints + beam step (beam.cu) ----
struct DevTables {
  int32_t offsets[3], sizes[3];
  const int32_t* table1; int32_t width1;
  const int32_t* table2; int32_t width2;
  const uint8_t* valid;
  int32_t root[3];
  const int32_t* first_tokens; int32_t n_first;
  int32_t newline, eos;
};

constexpr int MAX_BEAMS = 64;
constexpr int NSTEPS = 5;
constexpr int MAX_WIDTH = 256;
constexpr int TAIL_SPLITS = 16;

// Beam-search state in device memory (HF _beam_search running/finished sets).
struct BeamState {
  int32_t run_tok[MAX_BEAMS][NSTEPS];
  int32_t run_par[MAX_BEAMS][NSTEPS];
  float run_score[MAX_BEAMS];
  int32_t fin_tok[MAX_BEAMS][NSTEPS];
  int32_t fin_par[MAX_BEAMS][NSTEPS];
  float fin_score[MAX_BEAMS];
  int32_t fin_done[MAX_BEAMS];
  int32_t unsatisfied;      // is_early_stop_heuristic_unsatisfied
  int32_t finished_after;   // step after which the loop stopped (-1: running)
  int32_t anc[MAX_BEAMS][4];  // physical suffix row of each beam's slot
  int32_t next_tok[MAX_BEAMS];  // input token of the next forward
  int32_t prompt_tail[3];   // last three prompt tokens (step-0 lookup)
  // per step processed scores at the allowed columns (the only finite ones)
  int32_t cols[NSTEPS][MAX_BEAMS][MAX_WIDTH];
  float vals[NSTEPS][MAX_BEAMS][MAX_WIDTH];
  int32_t width[NSTEPS];
  int32_t same_rows[NSTEPS];  // 1: every beam row holds row 0's logits (step 0)
  float row_stats[MAX_BEAMS][4];  // max, log-sum, max2, log-sum2
  float part[MAX_BEAMS][TAIL_SPLITS][3];  // max, sum1, sum2 partials
};

struct DevResult {
  int32_t token_ids[MAX_BEAMS * NSTEPS];
  int32_t beam_indices[MAX_BEAMS * NSTEPS];
  float sequence_logp[MAX_BEAMS];
  float transition_logp[MAX_BEAMS * NSTEPS];
  uint32_t status;
  int32_t steps;
};

cudaError_t beam_init();
cudaError_t beam_reset(BeamState* st, const int32_t* ids_dev, const int32_t* L_dev, int beams,
                       cudaStream_t stream);
// Full step tail on logits [rows, V] (rows = 1 at step 0, otherwise beams).
// `users` consecutive beam states, each with `rows` logits rows (1 at step 0, else beams)
// With `lse` (the LM head's per-128-column-tile (max, sum exp) partials,
// [row][ceil(vocab / 128)]) the tail reads the logits once: two launches
// instead of four.
cudaError_t beam_step(BeamState* st, const float* logits, int rows, int vocab, int beams, int step,
                      const DevTables& tb, uint32_t* status, cudaStream_t stream, int users = 1,
                      const float2* lse = nullptr);
cudaError_t beam_finalize(const BeamState* st, int beams, DevResult* res, const uint32_t* status,
                          cudaStream_t stream, int users = 1);
cudaError_t beam_dense_scores(const BeamState* st, int step, int beams, int vocab, float* out,
                              cudaStream_t stream);
int lookup_width(const DevTables& tb, int step);
// Processor scratch: PROC_SPLITS (max, sum) partial pairs per row.
constexpr int PROC_SPLITS = 16;
constexpr int PROC_MAX_ROWS = 4096;
// Allocation-free variant: partials in a static device array of 256 rows.
constexpr int STATIC_PROC_MAX_ROWS = 256;
constexpr int STATIC_PROC_MAX_DEVICES = 64;
cudaError_t constraint_process_static(const DevTables& tb, int step, const int64_t* ids, int rows, int cols,
                                      const float* scores, float* out, int vocab, cudaStream_t stream);
cudaError_t constraint_lookup(const DevTables& tb, int step, const int64_t* ids, int rows, int cols,
                              int32_t* out, cudaStream_t stream);
cudaError_t constraint_process(const DevTables& tb, int step, const int64_t* ids, int rows, int cols,
                               const float* scores, float* out, int vocab, float* scratch,
                               cudaStream_t stream);

}  // namespace rtr
