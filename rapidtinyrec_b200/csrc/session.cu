// Session state and the C ABI (include/rtr_b200.h).
//
// Device layout of one session (one replica of the model on one GPU):
//   weights   embed [V,H]; per layer Wqkv [Hq*D+2*Hkv*D, H] (q, k, v rows),
//             bias [Hq*D+2*Hkv*D], Wo [H, Hq*D], Wgu [2I, H] (gate/up rows
//             interleaved in blocks of 16), Wd [H, I], two norms; final norm;
//             lm_head (aliases embed when tied)
//   prefix    [layers][K|V][Hkv][max_prefix][D]   one physical copy per request
//   suffix    [layers][K|V][4 slots][beams][Hkv][D]   written in place per step;
//             beams find their ancestors' slots through BeamState::anc
//   logits    [beams, V] fp32 (L2-resident between the LM head and the tail)
// A request is: prefill (eager launches, M = L rows) -> step-0 tail, then one
// CUDA graph holding decode steps 1..4 (forward + tail each) and the result
// copy; the prefix length lives in device memory so the graph serves every L.
#include <cuda_runtime.h>

#include <cmath>
#include <cstdio>
#include <cstring>
#include <string>
#include <cstdlib>
#include <map>
#include <utility>
#include <vector>

#include "../../include/rtr_b200.h"
#include "common.cuh"
#include "engine.h"

using namespace rtr;

struct LayerW {
  float *wqkv = nullptr, *bqkv = nullptr, *wo = nullptr, *wgu = nullptr, *wd = nullptr, *n_in = nullptr,
        *n_post = nullptr;
  // bf16 mode: the packed bf16 GEMM operands (no fp32 copies are kept)
  void *pqkv = nullptr, *po = nullptr, *pgu = nullptr, *pd = nullptr;
};

static constexpr int kTickets = 4096;  // split-K tickets: one per output tile
static constexpr int kMaxUsers = 8;

struct rtr_session {
  rtr_model_config cfg{};
  int device = 0, sms = 148;
  cudaStream_t stream = nullptr;
  bool own_stream = false;
  bool pdl = true;
  bool use_tc = true;  // tcgen05 GEMMs (RTR_GEMM=ffma selects the FFMA kernel)
  bool tc_wide = true;  // 128-row tcgen05 GEMM for M > 64 (RTR_TC_WIDE=0: the 64-row kernel only)
  // GEMM operand format of the fp32 tensor-core path: SPLIT_F16, the fp16-pair
  // kernel (default), or SPLIT_TF32, the 3xTF32 kernels (RTR_GEMM=tf32); every
  // activation producer writes its split in this format
  int xfmt = SPLIT_TF32;
  // RMSNorm folded into the GEMMs (fp32 tensor-core paths, hidden % 128 == 0;
  // RTR_NORM_FOLD=0 keeps the separate norm kernels): norm weights folded into the
  // packed q/k/v, gate/up and LM-head columns, row scales from partial sums of squares
  bool fold = false;
  float *x_big = nullptr, *x_small = nullptr, *ss = nullptr;  // split and partials of the residual stream
  int ss_ld = 0;
  // bf16 mode (RTR_DTYPE_BF16): bf16 weights, activations and KV; biases and
  // norm weights as bf16 values in fp32; logits in fp32.  The activation and
  // KV buffers below keep their float pointers and hold bf16 elements.
  bool bf16 = false;
  void* embed_bf = nullptr;      // bf16 [V][H] (embedding gather)
  void* lm_packed_bf = nullptr;  // packed bf16 LM head (the embedding when tied)
  // TMA descriptors keyed by (buffer, box rows): activations at 64/128 rows,
  // weights at 128 rows
  std::map<std::pair<const void*, int>, TensorMap> tmaps;
  std::map<const void*, float*> packed;  // tile-packed copy of each weight matrix
  std::string err;
  // weights
  float *embed = nullptr, *lm_head = nullptr, *norm_final = nullptr;
  std::vector<LayerW> layers;
  std::vector<void*> allocs;
  bool weights_loaded = false, tables_loaded = false;
  // rope
  float *rope_cos = nullptr, *rope_sin = nullptr;
  int rope_positions = 0;
  // tables
  DevTables tb{};
  int32_t *t1 = nullptr, *t2 = nullptr, *tfirst = nullptr;
  uint8_t* tvalid = nullptr;
  // KV and activations
  float *kv_prefix = nullptr, *kv_suffix = nullptr;
  TensorMap arena_map{};     // TMA map over the prefix arena (folded decode attention)
  // tensor-core decode attention: the prefix K / V as fp16 pairs, written by the prefill
  bool tc_attn = false;
  bool tc_prefill = false;  // prefill attention on the tensor cores (attn_tc.cu)
  uint16_t* vt_bf16 = nullptr;  // bf16 mode: V transposed per (user, layer, group) for the tensor-core attention
  bool tc_attn_bf16 = false;    // bf16 mode: decode attention on the tensor cores (attn_tc.cu)
  BfPrefillMaps pbmaps = {};
  __half* kvpair = nullptr;  // [K hi][K lo][V^T hi][V^T lo] planes
  AttnPairs pairs{};
  float2* lse = nullptr;     // LM head's per-tile (max, sum exp) partials: [tiles][B * max_users]
  bool lse_tail = false;     // decode step tails read the logits once (fp16-pair or bf16 LM head)
  bool folded_attn = false;
  float *x = nullptr, *h = nullptr, *qkv = nullptr, *q = nullptr, *attn = nullptr, *act = nullptr;
  // tf32 split (big = tf32(v), small = v - big) of the GEMM activation operands
  float *h_big = nullptr, *h_small = nullptr, *attn_big = nullptr, *attn_small = nullptr;
  float *act_big = nullptr, *act_small = nullptr;
  std::map<const void*, std::pair<float*, float*>> split_of;
  float *logits = nullptr, *ws = nullptr;
  float* proc_scratch = nullptr;  // [PROC_MAX_ROWS][PROC_SPLITS][2]
  size_t ws_floats = 0;
  int* tickets = nullptr;
  BeamState* beam = nullptr;
  DevResult* dres = nullptr;
  DevResult* hres = nullptr;  // pinned
  int32_t* d_ids = nullptr;
  int32_t* d_L = nullptr;
  int32_t* h_L = nullptr;     // pinned staging
  int32_t* h_ids = nullptr;   // pinned staging [max_prefix]
  uint32_t* d_status = nullptr;
  // request state
  int L = 0;
  int steps_done = -1;
  bool in_flight = false;
  // batched decode (rtr_session_create_batched): up to max_users users share each
  // decode step's GEMMs; user u has its own prefix arena, length, beam state and
  // result.  The per-step entry points serve user 0.
  int max_users = 1;
  int step_users = 1;        // users of the request in flight
  int cur_user = 0;          // the user whose prefill runs
  long prefix_user = 0;      // prefix-arena elements per user
  int Ls[kMaxUsers] = {};
  cudaGraphExec_t graphs[kMaxUsers + 1] = {};  // decode graph per batch size
  // counters (rtr_get_report)
  int64_t requests = 0, launches = 0, graph_kernels = 0;
  int64_t weight_bytes = 0, device_bytes = 0;
};

static std::string g_create_error;

static int fail(rtr_session* s, int code, const std::string& msg) {
  if (s) s->err = msg; else g_create_error = msg;
  return code;
}

#define CUDA_TRY(s, expr)                                                                 \
  do {                                                                                    \
    cudaError_t _e = (expr);                                                              \
    if (_e != cudaSuccess)                                                                \
      return fail((s), RTR_ERR_CUDA, std::string(#expr) + ": " + cudaGetErrorString(_e)); \
  } while (0)

static void drop_graphs(rtr_session* s) {
  for (auto& g : s->graphs)
    if (g) { cudaGraphExecDestroy(g); g = nullptr; }
}

template <typename T>
static cudaError_t dev_alloc(rtr_session* s, T** p, size_t count) {
  void* raw = nullptr;
  cudaError_t e = cudaMalloc(&raw, count * sizeof(T) + 256);
  if (e != cudaSuccess) return e;
  s->allocs.push_back(raw);
  s->device_bytes += (int64_t)(count * sizeof(T) + 256);
  *p = static_cast<T*>(raw);
  return cudaSuccess;
}

  // split-K tickets: one per output tile

static int beams_of(const rtr_session* s) { return s->cfg.num_beams; }
static int qkv_dim(const rtr_model_config& c) { return (c.heads + 2 * c.kv_heads) * c.head_dim; }

static void default_rope(const rtr_model_config& c, int n, std::vector<float>& cs, std::vector<float>& sn) {
  const int half = c.head_dim / 2;
  cs.resize((size_t)n * half);
  sn.resize((size_t)n * half);
  for (int i = 0; i < half; ++i) {
    const float expo = (float)(2 * i) / (float)c.head_dim;
    const float inv = (float)(1.0 / std::pow((double)c.rope_theta, (double)expo));
    for (int p = 0; p < n; ++p) {
      const float ang = inv * (float)p;
      cs[(size_t)p * half + i] = (float)std::cos((double)ang);
      sn[(size_t)p * half + i] = (float)std::sin((double)ang);
    }
  }
}

extern "C" {

const char* rtr_last_error(const rtr_session* s) { return s ? s->err.c_str() : g_create_error.c_str(); }

int rtr_session_create(const rtr_model_config* cfg, int device, rtr_session** out) {
  return rtr_session_create_batched(cfg, device, 1, out);
}

int rtr_session_create_batched(const rtr_model_config* cfg, int device, int32_t max_users, rtr_session** out) {
  if (!cfg || !out) return fail(nullptr, RTR_ERR_ARG, "null config or output pointer");
  if (max_users < 1 || max_users > kMaxUsers) return fail(nullptr, RTR_ERR_ARG, "max_users must be in [1, 8]");
  const rtr_model_config& c = *cfg;
  if (c.layers < 1 || c.hidden < 16 || c.heads < 1 || c.kv_heads < 1 || c.vocab < 16)
    return fail(nullptr, RTR_ERR_ARG, "non-positive model dimension");
  if (c.heads % c.kv_heads) return fail(nullptr, RTR_ERR_ARG, "heads must be a multiple of kv_heads");
  if (c.head_dim != 64 && c.head_dim != 128) return fail(nullptr, RTR_ERR_ARG, "head_dim must be 64 or 128");
  if (c.hidden % 16 || c.intermediate % 16 || (c.heads * c.head_dim) % 16)
    return fail(nullptr, RTR_ERR_ARG, "hidden, intermediate and heads*head_dim must be multiples of 16");
  if (c.num_beams < 1 || c.num_beams > MAX_BEAMS) return fail(nullptr, RTR_ERR_ARG, "num_beams must be in [1, 64]");
  if (c.max_prefix < 3 || c.max_prefix > 32768) return fail(nullptr, RTR_ERR_ARG, "max_prefix must be in [3, 32768]");
  if ((long)c.num_beams * c.vocab >= (1L << 32)) return fail(nullptr, RTR_ERR_ARG, "beams*vocab must fit 32 bits");
  if (c.dtype != RTR_DTYPE_F32 && c.dtype != RTR_DTYPE_BF16) return fail(nullptr, RTR_ERR_ARG, "unknown dtype");

  auto* s = new rtr_session();
  s->cfg = c;
  s->device = device;
  s->max_users = max_users;
  auto bail = [&](int code) {
    g_create_error = s->err;
    rtr_session_destroy(s);
    return code;
  };
#define CREATE_TRY(expr)                                                              \
  do {                                                                                \
    cudaError_t _e = (expr);                                                          \
    if (_e != cudaSuccess) {                                                          \
      s->err = std::string(#expr) + ": " + cudaGetErrorString(_e);                    \
      return bail(RTR_ERR_CUDA);                                                      \
    }                                                                                 \
  } while (0)
  CREATE_TRY(cudaSetDevice(device));
  CREATE_TRY(cudaDeviceGetAttribute(&s->sms, cudaDevAttrMultiProcessorCount, device));
  CREATE_TRY(cudaStreamCreateWithFlags(&s->stream, cudaStreamNonBlocking));
  s->own_stream = true;
  CREATE_TRY(gemm_init());
  CREATE_TRY(beam_init());
  CREATE_TRY(gemm_tc_init());
  CREATE_TRY(gemm_tc_wide_init());
  CREATE_TRY(attention_init());
  CREATE_TRY(attention_folded_init());
  CREATE_TRY(attention_tc_init());
  CREATE_TRY(gemm_bf16_init());
  CREATE_TRY(gemm_f16x2_init());
  bool tf32 = false;
  if (const char* g = std::getenv("RTR_GEMM")) {
    s->use_tc = std::strcmp(g, "ffma") != 0;
    tf32 = std::strcmp(g, "tf32") == 0;
  }
  if (const char* g = std::getenv("RTR_TC_WIDE")) s->tc_wide = std::strcmp(g, "0") != 0;
  s->fold = s->use_tc && c.dtype != RTR_DTYPE_BF16 && c.hidden % 128 == 0;
  if (const char* g = std::getenv("RTR_NORM_FOLD")) s->fold = s->fold && std::strcmp(g, "0") != 0;
  s->pdl = pdl_on(PDL_GEMM);
  s->bf16 = c.dtype == RTR_DTYPE_BF16;
  s->xfmt = s->use_tc && !s->bf16 && !tf32 ? SPLIT_F16 : SPLIT_TF32;
  if (s->bf16 && !s->use_tc) {
    s->err = "the bf16 mode runs on the tensor-core GEMMs only (unset RTR_GEMM)";
    return bail(RTR_ERR_ARG);
  }
  if (max_users > 1 && !s->use_tc) {
    s->err = "batched sessions run on the tensor-core GEMMs only (unset RTR_GEMM)";
    return bail(RTR_ERR_ARG);
  }

  const long H = c.hidden, V = c.vocab, I = c.intermediate, D = c.head_dim;
  const long qd = (long)c.heads * D, kvd = (long)c.kv_heads * D, qkvd = qkv_dim(c);
  const long B = c.num_beams, cap = c.max_prefix, U = max_users;
  const long M = cap > B * U ? cap : B * U;  // activation rows: a prefill or a batched decode step
  s->layers.resize(c.layers);
  if (!s->bf16) {
    CREATE_TRY(dev_alloc(s, &s->embed, V * H));
    for (auto& l : s->layers) {
      CREATE_TRY(dev_alloc(s, &l.wqkv, qkvd * H));
      CREATE_TRY(dev_alloc(s, &l.wo, H * qd));
      CREATE_TRY(dev_alloc(s, &l.wgu, 2 * I * H));
      CREATE_TRY(dev_alloc(s, &l.wd, H * I));
    }
    if (c.tied_embeddings) s->lm_head = s->embed;
    else CREATE_TRY(dev_alloc(s, &s->lm_head, V * H));
  } else {
    auto packed = [&](void** p, long rows, long cols) {
      uint16_t* q = nullptr;
      cudaError_t e = dev_alloc(s, &q, packed_weight_elems_bf16((int)rows, (int)cols));
      *p = q;
      return e;
    };
    uint16_t* eb = nullptr;
    CREATE_TRY(dev_alloc(s, &eb, (size_t)V * H));
    s->embed_bf = eb;
    for (auto& l : s->layers) {
      CREATE_TRY(packed(&l.pqkv, qkvd, H));
      CREATE_TRY(packed(&l.po, H, qd));
      CREATE_TRY(packed(&l.pgu, 2 * I, H));
      CREATE_TRY(packed(&l.pd, H, I));
    }
    CREATE_TRY(packed(&s->lm_packed_bf, V, H));
  }
  for (auto& l : s->layers) {
    CREATE_TRY(dev_alloc(s, &l.bqkv, qkvd));
    CREATE_TRY(dev_alloc(s, &l.n_in, H));
    CREATE_TRY(dev_alloc(s, &l.n_post, H));
  }
  CREATE_TRY(dev_alloc(s, &s->norm_final, H));
  s->weight_bytes = s->device_bytes;

  s->prefix_user = (long)c.layers * 2 * kvd * cap;
  CREATE_TRY(dev_alloc(s, &s->kv_prefix, (size_t)s->prefix_user * U));
  CREATE_TRY(dev_alloc(s, &s->kv_suffix, (size_t)c.layers * 2 * 4 * B * U * kvd));
  {
    // decode attention: the per-head kernel of attention.cu; RTR_ATTN=tc the
    // tensor-core kernel of attn_tc.cu (fp32 mode, prompts of up to 448
    // tokens), RTR_ATTN=folded the folded FFMA cluster kernel of
    // attn_decode.cu.  Both folded kernels read each KV group's prefix once
    // per 128 (beam, head) rows; on B200 neither beats the per-head kernel
    // inside a decode step (2.45 and 2.46 against 2.43 ms at 1.5B).
    const char* e = getenv("RTR_ATTN");
    const long arena_rows = s->prefix_user * U / D;
    s->tc_attn = e && strcmp(e, "tc") == 0 && s->use_tc && !s->bf16 &&
                 attention_tc_supported(c.heads, c.kv_heads, D, cap);
    // prefill attention: the tensor-core kernels of attn_tc.cu (fp32 mode with
    // the tensor-core projections, whose q/k/v epilogue writes the pair copies
    // they read; the bf16 mode), unless RTR_PREFILL_ATTN=ffma asks for the
    // FFMA kernel
    const char* pe = getenv("RTR_PREFILL_ATTN");
    s->tc_prefill = !(pe && strcmp(pe, "ffma") == 0) && (s->bf16 || s->use_tc) &&
                    attention_prefill_tc_supported(c.heads, c.kv_heads, D);
    // the bf16 decode attention: the tensor-core kernel unless RTR_ATTN=rows or
    // =folded names another one; it reads the prefix arena and V copy below
    s->tc_attn_bf16 = s->bf16 && !(e && (strcmp(e, "rows") == 0 || strcmp(e, "folded") == 0)) &&
                      attention_decode_tc_bf16_supported(c.heads, c.kv_heads, D);
    if (s->bf16 && (s->tc_prefill || s->tc_attn_bf16)) {
      const int pc = (cap + 63) / 64 * 64;
      const long vt_rows = (long)U * c.layers * c.kv_heads * D;
      CREATE_TRY(dev_alloc(s, &s->vt_bf16, (size_t)vt_rows * pc));
      CREATE_TRY(cudaMemset(s->vt_bf16, 0, (size_t)vt_rows * pc * sizeof(uint16_t)));
      s->pbmaps.pair_cap = pc;
      if (!make_tmap_bf16(&s->pbmaps.kmap, s->kv_prefix, arena_rows, D, D, 64) ||
          !make_tmap_bf16(&s->pbmaps.vmap, s->vt_bf16, vt_rows, pc, pc, D))
        return fail(nullptr, RTR_ERR_CUDA, "tensor map of the bf16 prefix arena / V copy");
    }
    if (s->tc_attn || (s->tc_prefill && !s->bf16)) {
      const int pc = (cap + 63) / 64 * 64;
      const long plane = (long)U * c.layers * c.kv_heads * pc * D;  // halfs per plane (K and V^T alike)
      CREATE_TRY(dev_alloc(s, &s->kvpair, (size_t)4 * plane));
      CREATE_TRY(cudaMemset(s->kvpair, 0, (size_t)4 * plane * sizeof(__half)));
      AttnPairs& ap = s->pairs;
      ap.pair_cap = pc;
      ap.kplane = plane / D;                            // K rows per plane
      ap.kuser = (long)c.layers * c.kv_heads * pc;
      ap.vplane = plane / pc;                           // V^T rows per plane
      ap.vuser = (long)c.layers * c.kv_heads * D;
      if (!make_tmap_f16(&ap.kmap, s->kvpair, 2 * ap.kplane, D, D, 64) ||
          !make_tmap_f16(&ap.vmap, s->kvpair + 2 * plane, 2 * ap.vplane, pc, pc, D))
        return fail(nullptr, RTR_ERR_CUDA, "tensor map of the K / V pair copies");
    }
    s->folded_attn = e && strcmp(e, "folded") == 0 && attention_folded_supported(c.heads, c.kv_heads, D, s->bf16) &&
                     (s->bf16 ? make_tmap_bf16(&s->arena_map, s->kv_prefix, arena_rows, D, D, 32)
                              : make_tmap_f32(&s->arena_map, s->kv_prefix, arena_rows, D, D, 32));
  }
  CREATE_TRY(dev_alloc(s, &s->x, M * H));
  CREATE_TRY(dev_alloc(s, &s->h, M * H));
  CREATE_TRY(dev_alloc(s, &s->qkv, M * qkvd));
  CREATE_TRY(dev_alloc(s, &s->q, M * qd));
  CREATE_TRY(dev_alloc(s, &s->attn, M * qd));
  CREATE_TRY(dev_alloc(s, &s->act, M * I));
  if (!s->bf16) {
    CREATE_TRY(dev_alloc(s, &s->h_big, M * H));
    CREATE_TRY(dev_alloc(s, &s->h_small, M * H));
    CREATE_TRY(dev_alloc(s, &s->attn_big, M * qd));
    CREATE_TRY(dev_alloc(s, &s->attn_small, M * qd));
    CREATE_TRY(dev_alloc(s, &s->act_big, M * I));
    CREATE_TRY(dev_alloc(s, &s->act_small, M * I));
  }
  if (s->fold) {
    CREATE_TRY(dev_alloc(s, &s->x_big, M * H));
    CREATE_TRY(dev_alloc(s, &s->x_small, M * H));
    s->ss_ld = (int)M;
    CREATE_TRY(dev_alloc(s, &s->ss, (H / 128) * M));
  }
  CREATE_TRY(dev_alloc(s, &s->logits, B * U * V));
  {
    // the fp16-pair and bf16 LM heads leave the first log-softmax's partials
    // (RTR_TAIL=passes: three passes over the logits instead)
    const char* e = getenv("RTR_TAIL");
    s->lse_tail = s->use_tc && (s->xfmt == SPLIT_F16 || s->bf16) && !(e && strcmp(e, "passes") == 0);
    if (s->lse_tail) CREATE_TRY(dev_alloc(s, &s->lse, (size_t)((V + 127) / 128) * B * U));
  }
  long max_n = qkvd;
  if (H > max_n) max_n = H;
  if (2 * I > max_n) max_n = 2 * I;
  s->ws_floats = gemm_workspace_floats(64, (int)max_n, s->sms);
  // the tensor-core GEMMs split K only while tiles x splits <= SMs: a full set of
  // 128 x 128 partial tiles (the 128-row kernel) must fit, or a GEMM would run
  // with fewer splits than its 64-row twin and round differently
  if (s->ws_floats < (size_t)s->sms * 128 * 128) s->ws_floats = (size_t)s->sms * 128 * 128;
  CREATE_TRY(dev_alloc(s, &s->ws, s->ws_floats));
  CREATE_TRY(dev_alloc(s, &s->tickets, kTickets));
  CREATE_TRY(dev_alloc(s, &s->proc_scratch, (size_t)PROC_MAX_ROWS * PROC_SPLITS * 2));
  CREATE_TRY(cudaMemset(s->tickets, 0, kTickets * sizeof(int)));
  CREATE_TRY(dev_alloc(s, &s->beam, U));
  CREATE_TRY(cudaMemset(s->beam, 0, U * sizeof(BeamState)));
  CREATE_TRY(dev_alloc(s, &s->dres, U));
  CREATE_TRY(dev_alloc(s, &s->d_ids, cap));
  CREATE_TRY(dev_alloc(s, &s->d_L, U));
  CREATE_TRY(dev_alloc(s, &s->d_status, 1));
  CREATE_TRY(cudaMemset(s->d_status, 0, sizeof(uint32_t)));
  CREATE_TRY(cudaMallocHost(&s->hres, U * sizeof(DevResult)));
  CREATE_TRY(cudaMallocHost(&s->h_L, U * sizeof(int32_t)));
  CREATE_TRY(cudaMallocHost(&s->h_ids, U * cap * sizeof(int32_t)));

  s->rope_positions = (int)cap + 8;
  CREATE_TRY(dev_alloc(s, &s->rope_cos, (size_t)s->rope_positions * D / 2));
  CREATE_TRY(dev_alloc(s, &s->rope_sin, (size_t)s->rope_positions * D / 2));
  std::vector<float> cs, sn;
  default_rope(c, s->rope_positions, cs, sn);
  CREATE_TRY(cudaMemcpy(s->rope_cos, cs.data(), cs.size() * sizeof(float), cudaMemcpyHostToDevice));
  CREATE_TRY(cudaMemcpy(s->rope_sin, sn.data(), sn.size() * sizeof(float), cudaMemcpyHostToDevice));
  if (s->bf16) {  // a bf16 model rotates with bf16 cos/sin
    CREATE_TRY(round_to_bf16(s->rope_cos, (int64_t)cs.size(), 0));
    CREATE_TRY(round_to_bf16(s->rope_sin, (int64_t)sn.size(), 0));
    CREATE_TRY(cudaDeviceSynchronize());
  }

  // TMA descriptors of the GEMM activation operands: the big and small halves
  // (bf16 mode: the bf16 buffers themselves)
  struct Act { const float* v; float* big; float* small; long width; };
  const Act acts[4] = {{s->h, s->h_big, s->h_small, H}, {s->attn, s->attn_big, s->attn_small, qd},
                       {s->act, s->act_big, s->act_small, I}, {s->x, s->x_big, s->x_small, H}};
  for (const auto& a : acts) {
    if (a.v == s->x && !s->fold) continue;
    if (s->bf16) {
      TensorMap m;
      if (!make_tmap_bf16(&m, a.v, M, a.width, a.width, 64)) {
        s->err = "cuTensorMapEncodeTiled failed for a bf16 activation buffer";
        return bail(RTR_ERR_CUDA);
      }
      s->tmaps[{a.v, 64}] = m;
      continue;
    }
    s->split_of[a.v] = {a.big, a.small};
    for (const float* half : {a.big, a.small}) {
      TensorMap m;
      const bool ok = s->xfmt == SPLIT_F16 ? make_tmap_f16(&m, half, M, a.width, a.width, 64)
                                           : make_tmap_f32(&m, half, M, a.width, a.width, 64);
      if (!ok) {
        s->err = "cuTensorMapEncodeTiled failed for an activation buffer";
        return bail(RTR_ERR_CUDA);
      }
      s->tmaps[{half, 64}] = m;
    }
  }
#undef CREATE_TRY
  *out = s;
  return RTR_OK;
}

int rtr_session_destroy(rtr_session* s) {
  if (!s) return RTR_OK;
  cudaSetDevice(s->device);
  for (auto& g : s->graphs)
    if (g) cudaGraphExecDestroy(g);
  for (void* p : s->allocs) cudaFree(p);
  if (s->tvalid) cudaFree(s->tvalid);
  if (s->t1) cudaFree(s->t1);
  if (s->t2) cudaFree(s->t2);
  if (s->tfirst) cudaFree(s->tfirst);
  if (s->hres) cudaFreeHost(s->hres);
  if (s->h_L) cudaFreeHost(s->h_L);
  if (s->h_ids) cudaFreeHost(s->h_ids);
  if (s->own_stream && s->stream) cudaStreamDestroy(s->stream);
  delete s;
  return RTR_OK;
}

int rtr_set_stream(rtr_session* s, void* stream) {
  if (!s) return RTR_ERR_ARG;
  CUDA_TRY(s, cudaSetDevice(s->device));
  drop_graphs(s);
  if (s->own_stream) { cudaStreamDestroy(s->stream); s->own_stream = false; }
  if (stream) {
    s->stream = static_cast<cudaStream_t>(stream);
  } else {
    CUDA_TRY(s, cudaStreamCreateWithFlags(&s->stream, cudaStreamNonBlocking));
    s->own_stream = true;
  }
  return RTR_OK;
}

int rtr_load_rope(rtr_session* s, const float* cos_host, const float* sin_host, int32_t n_positions) {
  if (!s || !cos_host || !sin_host) return RTR_ERR_ARG;
  if (n_positions < s->rope_positions)
    return fail(s, RTR_ERR_ARG, "rope table must cover max_prefix + 8 positions");
  const size_t bytes = (size_t)s->rope_positions * s->cfg.head_dim / 2 * sizeof(float);
  CUDA_TRY(s, cudaSetDevice(s->device));
  CUDA_TRY(s, cudaMemcpy(s->rope_cos, cos_host, bytes, cudaMemcpyHostToDevice));
  CUDA_TRY(s, cudaMemcpy(s->rope_sin, sin_host, bytes, cudaMemcpyHostToDevice));
  if (s->bf16) {  // a bf16 model rotates with bf16 cos/sin (cos/sin .to(bfloat16))
    CUDA_TRY(s, round_to_bf16(s->rope_cos, (int64_t)(bytes / sizeof(float)), 0));
    CUDA_TRY(s, round_to_bf16(s->rope_sin, (int64_t)(bytes / sizeof(float)), 0));
    CUDA_TRY(s, cudaDeviceSynchronize());
  }
  return RTR_OK;
}

// bf16 mode: every matrix is staged once in fp32 on the device, rounded to
// bf16 and packed into the GEMM's tile blocks; biases and norm weights are
// rounded in place (a bf16 model's parameters).
static int load_weights_bf16(rtr_session* s, const void* const* tensors, int32_t src_on_device) {
  const auto& c = s->cfg;
  const cudaMemcpyKind kind = src_on_device ? cudaMemcpyDeviceToDevice : cudaMemcpyHostToDevice;
  const size_t H = c.hidden, V = c.vocab, I = c.intermediate, D = c.head_dim;
  const size_t qd = c.heads * D, kvd = c.kv_heads * D, qkvd = qd + 2 * kvd;
  const size_t f = sizeof(float);
  size_t most = V * H;
  for (size_t n : {qkvd * H, H * qd, 2 * I * H, H * I}) most = n > most ? n : most;
  float* stage = nullptr;
  CUDA_TRY(s, cudaMalloc(&stage, most * f));
  auto cp = [&](void* dst, const void* src, size_t n) { return cudaMemcpy(dst, src, n * f, kind); };
  auto pack = [&](void* dst, size_t rows, size_t cols) -> cudaError_t {
    cudaError_t e = pack_weight_tiles_bf16(stage, (int)rows, (int)cols, dst, 0);
    if (e != cudaSuccess) return e;
    TensorMap m;
    if (!make_tmap_packed_bf16(&m, dst, (int)rows, (int)cols)) return cudaErrorInvalidValue;
    s->tmaps[{dst, 128}] = m;
    return cudaDeviceSynchronize();  // the stage is reused by the next matrix
  };
  auto params = [&](float* dst, const void* src, size_t n) -> cudaError_t {
    cudaError_t e = cp(dst, src, n);
    return e != cudaSuccess ? e : round_to_bf16(dst, (int64_t)n, 0);
  };
  cudaError_t e = cp(stage, tensors[0], V * H);
  if (e == cudaSuccess) e = f32_to_bf16(stage, s->embed_bf, (int64_t)(V * H), 0);
  if (e == cudaSuccess && c.tied_embeddings) e = pack(s->lm_packed_bf, V, H);
  for (int l = 0; l < c.layers && e == cudaSuccess; ++l) {
    const void* const* t = tensors + 1 + 12 * l;
    LayerW& w = s->layers[l];
    e = cp(stage, t[0], qd * H);                                        // q, k, v rows
    if (e == cudaSuccess) e = cp(stage + qd * H, t[2], kvd * H);
    if (e == cudaSuccess) e = cp(stage + (qd + kvd) * H, t[4], kvd * H);
    if (e == cudaSuccess) e = pack(w.pqkv, qkvd, H);
    if (e == cudaSuccess) e = params(w.bqkv, t[1], qd);
    if (e == cudaSuccess) e = params(w.bqkv + qd, t[3], kvd);
    if (e == cudaSuccess) e = params(w.bqkv + qd + kvd, t[5], kvd);
    if (e == cudaSuccess) e = cp(stage, t[6], H * qd);
    if (e == cudaSuccess) e = pack(w.po, H, qd);
    // gate/up interleaved in blocks of 16 rows
    if (e == cudaSuccess) e = cudaMemcpy2D(stage, 32 * H * f, t[7], 16 * H * f, 16 * H * f, I / 16, kind);
    if (e == cudaSuccess) e = cudaMemcpy2D(stage + 16 * H, 32 * H * f, t[8], 16 * H * f, 16 * H * f, I / 16, kind);
    if (e == cudaSuccess) e = pack(w.pgu, 2 * I, H);
    if (e == cudaSuccess) e = cp(stage, t[9], H * I);
    if (e == cudaSuccess) e = pack(w.pd, H, I);
    if (e == cudaSuccess) e = params(w.n_in, t[10], H);
    if (e == cudaSuccess) e = params(w.n_post, t[11], H);
  }
  if (e == cudaSuccess) e = params(s->norm_final, tensors[1 + 12 * c.layers], H);
  if (e == cudaSuccess && !c.tied_embeddings) {
    e = cp(stage, tensors[2 + 12 * c.layers], V * H);
    if (e == cudaSuccess) e = pack(s->lm_packed_bf, V, H);
  }
  if (e == cudaSuccess) e = cudaDeviceSynchronize();
  cudaFree(stage);
  if (e != cudaSuccess) return fail(s, RTR_ERR_CUDA, std::string("bf16 weight load: ") + cudaGetErrorString(e));
  s->weights_loaded = true;
  return RTR_OK;
}

int rtr_load_weights(rtr_session* s, const void* const* tensors, int32_t n_tensors, int32_t src_dtype,
                     int32_t src_on_device) {
  if (!s || !tensors) return RTR_ERR_ARG;
  const auto& c = s->cfg;
  const int expect = 1 + 12 * c.layers + 1 + (c.tied_embeddings ? 0 : 1);
  if (n_tensors != expect) return fail(s, RTR_ERR_ARG, "expected " + std::to_string(expect) + " weight tensors");
  if (src_dtype != RTR_DTYPE_F32) return fail(s, RTR_ERR_ARG, "weights must be float32 for this build");
  for (int i = 0; i < n_tensors; ++i)
    if (!tensors[i]) return fail(s, RTR_ERR_ARG, "null weight tensor " + std::to_string(i));
  CUDA_TRY(s, cudaSetDevice(s->device));
  if (s->bf16) return load_weights_bf16(s, tensors, src_on_device);
  const cudaMemcpyKind kind = src_on_device ? cudaMemcpyDeviceToDevice : cudaMemcpyHostToDevice;
  const size_t H = c.hidden, V = c.vocab, I = c.intermediate, D = c.head_dim;
  const size_t qd = c.heads * D, kvd = c.kv_heads * D;
  const size_t f = sizeof(float);
  auto cp = [&](void* dst, const void* src, size_t n) { return cudaMemcpy(dst, src, n * f, kind); };
  CUDA_TRY(s, cp(s->embed, tensors[0], V * H));
  for (int l = 0; l < c.layers; ++l) {
    const void* const* t = tensors + 1 + 12 * l;
    LayerW& w = s->layers[l];
    CUDA_TRY(s, cp(w.wqkv, t[0], qd * H));
    CUDA_TRY(s, cp(w.bqkv, t[1], qd));
    CUDA_TRY(s, cp(w.wqkv + qd * H, t[2], kvd * H));
    CUDA_TRY(s, cp(w.bqkv + qd, t[3], kvd));
    CUDA_TRY(s, cp(w.wqkv + (qd + kvd) * H, t[4], kvd * H));
    CUDA_TRY(s, cp(w.bqkv + qd + kvd, t[5], kvd));
    CUDA_TRY(s, cp(w.wo, t[6], H * qd));
    // gate/up interleaved in blocks of 16 rows
    CUDA_TRY(s, cudaMemcpy2D(w.wgu, 32 * H * f, t[7], 16 * H * f, 16 * H * f, I / 16, kind));
    CUDA_TRY(s, cudaMemcpy2D(w.wgu + 16 * H, 32 * H * f, t[8], 16 * H * f, 16 * H * f, I / 16, kind));
    CUDA_TRY(s, cp(w.wd, t[9], H * I));
    CUDA_TRY(s, cp(w.n_in, t[10], H));
    CUDA_TRY(s, cp(w.n_post, t[11], H));
  }
  CUDA_TRY(s, cp(s->norm_final, tensors[1 + 12 * c.layers], H));
  if (!c.tied_embeddings) CUDA_TRY(s, cp(s->lm_head, tensors[2 + 12 * c.layers], V * H));
  CUDA_TRY(s, cudaDeviceSynchronize());
  // Tensor-core GEMM operands: every weight matrix packed into tile-contiguous
  // blocks (allocated once), with its TMA descriptor keyed by the original matrix
  if (s->use_tc) {
    auto wmap = [&](const float* w, long rows, long cols, const float* col_scale = nullptr) -> cudaError_t {
      const bool f16 = s->xfmt == SPLIT_F16;
      float* packed = nullptr;
      auto it = s->packed.find(w);
      if (it == s->packed.end()) {
        const size_t floats = f16 ? packed_weight_elems_f16x2((int)rows, (int)cols) / 2
                                  : packed_weight_floats((int)rows, (int)cols);
        cudaError_t e = dev_alloc(s, &packed, floats);
        if (e != cudaSuccess) return e;
        s->packed[w] = packed;
      } else {
        packed = it->second;
      }
      cudaError_t e = f16 ? pack_weight_tiles_f16x2(w, (int)rows, (int)cols, packed, 0, col_scale)
                          : pack_weight_tiles(w, (int)rows, (int)cols, packed, 0, col_scale);
      if (e != cudaSuccess) return e;
      TensorMap m;
      if (!(f16 ? make_tmap_packed_f16x2(&m, packed, (int)rows, (int)cols)
                : make_tmap_packed(&m, packed, (int)rows, (int)cols)))
        return cudaErrorInvalidValue;
      s->tmaps[{w, 128}] = m;
      return cudaSuccess;
    };
    // with the norm fold, the LM head, q/k/v and gate/up carry their norm's weight
    CUDA_TRY(s, wmap(s->lm_head, V, H, s->fold ? s->norm_final : nullptr));
    for (int l = 0; l < c.layers; ++l) {
      const LayerW& w = s->layers[l];
      CUDA_TRY(s, wmap(w.wqkv, qd + 2 * kvd, H, s->fold ? w.n_in : nullptr));
      CUDA_TRY(s, wmap(w.wo, H, qd));
      CUDA_TRY(s, wmap(w.wgu, 2 * I, H, s->fold ? w.n_post : nullptr));
      CUDA_TRY(s, wmap(w.wd, H, I));
    }
    CUDA_TRY(s, cudaDeviceSynchronize());
  }
  s->weights_loaded = true;
  return RTR_OK;
}

int rtr_load_constraints(rtr_session* s, const rtr_constraint_tables* t) {
  if (!s || !t) return RTR_ERR_ARG;
  const auto& c = s->cfg;
  long prod = 1;
  for (int i = 0; i < 3; ++i) {
    if (t->sizes[i] < 1) return fail(s, RTR_ERR_ARG, "SID level sizes must be positive");
    prod *= t->sizes[i];
  }
  if (prod > 100000000L) return fail(s, RTR_ERR_ARG, "Dense SID-validity table too large for this implementation");
  if (t->width1 < 1 || t->width1 > MAX_WIDTH || t->width2 < 1 || t->width2 > MAX_WIDTH ||
      t->n_first < 1 || t->n_first > MAX_WIDTH)
    return fail(s, RTR_ERR_ARG, "lookup widths must be in [1, 256]");
  if (!t->table1 || !t->table2 || !t->valid || !t->first_tokens) return fail(s, RTR_ERR_ARG, "null table");
  auto in_vocab = [&](int v) { return v >= 0 && v < c.vocab; };
  if (!in_vocab(t->newline) || !in_vocab(t->eos)) return fail(s, RTR_ERR_ARG, "newline/eos outside the vocabulary");
  // every row: sorted unique tokens, then repeats of its first token (gpu_constraints.py:51-54)
  auto check_rows = [&](const int32_t* tab, long rows, int w) -> bool {
    for (long r = 0; r < rows; ++r) {
      const int32_t* row = tab + r * w;
      bool pad = false;
      for (int j = 0; j < w; ++j) {
        if (!in_vocab(row[j])) return false;
        if (j == 0) continue;
        if (row[j] == row[0]) pad = true;
        else if (pad || row[j] <= row[j - 1]) return false;
      }
    }
    return true;
  };
  const long rows1 = t->sizes[0], rows2 = (long)t->sizes[0] * t->sizes[1];
  if (!check_rows(t->table1, rows1, t->width1) || !check_rows(t->table2, rows2, t->width2) ||
      !check_rows(t->first_tokens, 1, t->n_first))
    return fail(s, RTR_ERR_ARG, "table rows must be sorted unique tokens padded with their first token");
  CUDA_TRY(s, cudaSetDevice(s->device));
  if (s->t1) { cudaFree(s->t1); cudaFree(s->t2); cudaFree(s->tfirst); cudaFree(s->tvalid); }
  CUDA_TRY(s, cudaMalloc(&s->t1, rows1 * t->width1 * sizeof(int32_t)));
  CUDA_TRY(s, cudaMalloc(&s->t2, rows2 * t->width2 * sizeof(int32_t)));
  CUDA_TRY(s, cudaMalloc(&s->tfirst, t->n_first * sizeof(int32_t)));
  CUDA_TRY(s, cudaMalloc(&s->tvalid, prod));
  CUDA_TRY(s, cudaMemcpy(s->t1, t->table1, rows1 * t->width1 * sizeof(int32_t), cudaMemcpyHostToDevice));
  CUDA_TRY(s, cudaMemcpy(s->t2, t->table2, rows2 * t->width2 * sizeof(int32_t), cudaMemcpyHostToDevice));
  CUDA_TRY(s, cudaMemcpy(s->tfirst, t->first_tokens, t->n_first * sizeof(int32_t), cudaMemcpyHostToDevice));
  CUDA_TRY(s, cudaMemcpy(s->tvalid, t->valid, prod, cudaMemcpyHostToDevice));
  DevTables& d = s->tb;
  for (int i = 0; i < 3; ++i) { d.offsets[i] = t->offsets[i]; d.sizes[i] = t->sizes[i]; d.root[i] = t->root[i]; }
  d.table1 = s->t1; d.width1 = t->width1;
  d.table2 = s->t2; d.width2 = t->width2;
  d.valid = s->tvalid;
  d.first_tokens = s->tfirst; d.n_first = t->n_first;
  d.newline = t->newline; d.eos = t->eos;
  drop_graphs(s);
  s->tables_loaded = true;
  return RTR_OK;
}

}  // extern "C"

// ------------------------------------------------------------------ forward
// Projection GEMM on the split of activation buffer A and the weight matrix W:
// the fp16-pair tcgen05 kernel, the 3xTF32 ones (RTR_GEMM=tf32) or the FFMA
// kernel (RTR_GEMM=ffma).
static cudaError_t gemm(rtr_session* s, const float* A, int lda, const float* W, float* C, int ldc,
                        const float* bias, int M, int N, int K, int epi, const RopeArgs* rope = nullptr,
                        const NormFold* fold = nullptr, float2* lse = nullptr) {
  if (s->use_tc) {
    auto sp = s->split_of.find(A);
    if (sp == s->split_of.end()) return cudaErrorInvalidValue;
    auto xb = s->tmaps.find({sp->second.first, 64});
    auto xs = s->tmaps.find({sp->second.second, 64});
    auto w = s->tmaps.find({W, 128});
    if (xb == s->tmaps.end() || xs == s->tmaps.end() || w == s->tmaps.end()) return cudaErrorInvalidValue;
    float* cb = nullptr;
    float* cs = nullptr;
    if (epi == EPI_SWIGLU || (fold && fold->ss_out)) {
      auto out = s->split_of.find(C);
      if (out == s->split_of.end()) return cudaErrorInvalidValue;
      cb = out->second.first;
      cs = out->second.second;
    }
    if (s->xfmt == SPLIT_F16)
      return gemm_f16x2(w->second, xb->second, xs->second, C, cb, cs, ldc, bias, M, N, K, epi, s->ws, s->ws_floats,
                        s->tickets, kTickets, s->d_status, s->sms, s->stream, s->pdl, rope, fold, lse,
                        (s->cfg.vocab + 127) / 128);
    // more than 64 rows (the prefill): one 128-row MMA per instruction instead of two 64-row ones
    if (M > 64 && s->tc_wide)
      return gemm_tc_wide(w->second, xb->second, xs->second, C, cb, cs, ldc, bias, M, N, K, epi, s->ws,
                          s->ws_floats, s->tickets, kTickets, s->d_status, s->sms, s->stream, s->pdl, rope, fold);
    return gemm_tc(w->second, xb->second, xs->second, C, cb, cs, ldc, bias, M, N, K, epi, s->ws, s->ws_floats,
                   s->tickets, kTickets, s->d_status, s->sms, s->stream, s->pdl, rope, fold);
  }
  return gemm_f32(A, lda, W, C, ldc, bias, M, N, K, epi, s->ws, s->ws_floats, s->tickets, s->sms,
                  s->stream, s->pdl);
}

#define FWD_TRY(expr)                      \
  do {                                     \
    cudaError_t _e = (expr);               \
    if (_e != cudaSuccess) return _e;      \
  } while (0)

// bf16 mode: projection GEMM of the bf16 activation buffer X (its TMA map)
// against a packed bf16 weight.
static cudaError_t gemm16(rtr_session* s, const float* X, const void* Wp, void* C, int ldc, const float* bias, int M,
                          int N, int K, int epi, const RopeArgs* rope = nullptr, float2* lse = nullptr) {
  auto x = s->tmaps.find({X, 64});
  auto w = s->tmaps.find({Wp, 128});
  if (x == s->tmaps.end() || w == s->tmaps.end()) return cudaErrorInvalidValue;
  return gemm_bf16(w->second, x->second, C, ldc, bias, M, N, K, epi, s->ws, s->ws_floats, s->tickets, kTickets,
                   s->d_status, s->sms, s->stream, s->pdl, rope, lse, (s->cfg.vocab + 127) / 128, s->tc_wide);
}

// The prefill of user cur_user also writes layer l's K / V as fp16 pairs for
// the tensor-core decode attention.
static void set_pair_copies(const rtr_session* s, RopeArgs& ra, int l) {
  if (s->bf16 || (!s->tc_attn && !s->tc_prefill)) return;
  const auto& c = s->cfg;
  const AttnPairs& ap = s->pairs;
  const long lg = ((long)s->cur_user * c.layers + l) * c.kv_heads;
  const long plane = ap.kplane * c.head_dim;
  __half* k = s->kvpair + lg * ap.pair_cap * c.head_dim;
  __half* v = s->kvpair + 2 * plane + lg * c.head_dim * ap.pair_cap;
  ra.kpair_hi = k;
  ra.kpair_lo = k + plane;
  ra.vtpair_hi = v;
  ra.vtpair_lo = v + plane;
  ra.pair_cap = ap.pair_cap;
}

// Prefill attention of layer l over the M prompt rows of user cur_user: the
// tensor-core kernel (from the pair copies the q/k/v epilogue just wrote) or
// the FFMA kernel of attention.cu.
static cudaError_t prefill_attention(rtr_session* s, int l, const float* kp, const float* vp, int M, float scale) {
  const auto& c = s->cfg;
  if (s->tc_prefill) {
    AttnPairs ap = s->pairs;
    ap.krow0 = (long)l * c.kv_heads * ap.pair_cap;
    ap.vrow0 = (long)l * c.kv_heads * c.head_dim;
    return attention_prefill_tc(ap, s->cur_user, s->q, s->attn, s->attn_big, s->attn_small, M, c.heads, c.kv_heads,
                                c.head_dim, scale, s->d_status, s->stream, s->xfmt);
  }
  return attention_prefill(s->q, kp, vp, s->attn, s->attn_big, s->attn_small, M, c.max_prefix, c.heads, c.kv_heads,
                           c.head_dim, scale, false, s->stream, s->xfmt);
}

// Decode attention of layer l: the per-head kernel, the tensor-core kernel
// (RTR_ATTN=tc) or the folded cluster kernel (RTR_ATTN=folded).
static cudaError_t decode_attention(rtr_session* s, int l, const void* kp, const void* vp, const void* ks,
                                    const void* vs, int t, float* ob, float* os, float scale, const DecodeUsers& du) {
  const auto& c = s->cfg;
  const int D = c.head_dim;
  if (s->tc_attn_bf16)
    return attention_decode_tc_bf16(s->pbmaps, l, c.layers, s->q, ks, vs, &s->beam->anc[0][0], s->d_L, t, s->attn,
                                    beams_of(s), c.max_prefix, c.heads, c.kv_heads, D, scale, s->d_status, s->stream,
                                    du);
  if (s->tc_attn) {
    AttnPairs ap = s->pairs;
    ap.krow0 = (long)l * c.kv_heads * ap.pair_cap;
    ap.vrow0 = (long)l * c.kv_heads * D;
    return attention_decode_tc(ap, s->q, static_cast<const float*>(ks), static_cast<const float*>(vs),
                               &s->beam->anc[0][0], s->d_L, t, s->attn, ob, os, beams_of(s), c.max_prefix, c.heads,
                               c.kv_heads, D, scale, s->d_status, s->stream, du, s->xfmt);
  }
  if (s->folded_attn) {
    const long esz = s->bf16 ? 2 : 4;
    const char* base = reinterpret_cast<const char*>(s->kv_prefix);
    const long krow0 = (long)(reinterpret_cast<const char*>(kp) - base) / esz / D;
    const long vrow0 = (long)(reinterpret_cast<const char*>(vp) - base) / esz / D;
    return attention_decode_folded(s->arena_map, krow0, vrow0, s->prefix_user / D, s->q, ks, vs,
                                   &s->beam->anc[0][0], s->d_L, t, s->attn, ob, os, beams_of(s), c.max_prefix,
                                   c.heads, c.kv_heads, D, scale, s->d_status, s->bf16, s->stream, du, s->xfmt);
  }
  return attention_decode(s->q, kp, vp, ks, vs, &s->beam->anc[0][0], s->d_L, t, s->attn, ob, os, beams_of(s),
                          c.max_prefix, c.heads, c.kv_heads, D, scale, s->d_status, s->bf16, s->stream, du, s->xfmt);
}

// The forward of the bf16 mode: the same launches as the fp32 forward with
// bf16 activations, KV and weights (the reference's bf16-experimental model).
static cudaError_t forward_bf16(rtr_session* s, int t) {
  const auto& c = s->cfg;
  const int H = c.hidden, V = c.vocab, I = c.intermediate, D = c.head_dim;
  const int qd = c.heads * D, kvd = c.kv_heads * D, qkvd = qkv_dim(c);
  const int B = beams_of(s), cap = c.max_prefix;
  // t = 0: user cur_user's prefill; t >= 1: one decode step of step_users users
  const int n = s->step_users, RB = B * s->max_users;
  const int M = t == 0 ? s->Ls[s->cur_user] : B * n;
  const long pre_off = t == 0 ? (long)s->cur_user * s->prefix_user : 0;
  const DecodeUsers du{n, s->prefix_user, (int)(sizeof(BeamState) / sizeof(int32_t))};
  const float scale = (float)std::pow((double)D, -0.5);
  cudaStream_t st = s->stream;
  const int32_t* ids = t == 0 ? s->d_ids : &s->beam->next_tok[0];
  const int id_rows = t == 0 ? 0 : B;  // decode: user m / B's beam m % B
  const long id_stride = (long)(sizeof(BeamState) / sizeof(int32_t));
  uint16_t* kvp = reinterpret_cast<uint16_t*>(s->kv_prefix) + pre_off;  // bf16 elements
  uint16_t* kvs = reinterpret_cast<uint16_t*>(s->kv_suffix);
  FWD_TRY(embed_rows_bf16(ids, 1, M, s->embed_bf, V, H, s->x, s->d_status, st, id_rows, id_stride));
  for (int l = 0; l < c.layers; ++l) {
    const LayerW& w = s->layers[l];
    uint16_t* kp = kvp + (size_t)l * 2 * kvd * cap;
    uint16_t* vp = kp + (size_t)kvd * cap;
    uint16_t* ks = kvs + (size_t)l * 2 * 4 * RB * kvd;
    uint16_t* vs = ks + (size_t)4 * RB * kvd;
    const size_t slot = t == 0 ? 0 : (size_t)(t - 1) * B * n * kvd;
    FWD_TRY(rms_norm_rows_bf16(s->x, w.n_in, s->h, M, H, c.rms_eps, st));
    RopeArgs ra{s->rope_cos, s->rope_sin, s->rope_positions, c.heads, c.kv_heads, D, s->q,
                reinterpret_cast<float*>(t == 0 ? kp : ks + slot),
                reinterpret_cast<float*>(t == 0 ? vp : vs + slot), cap, t == 0 ? -1 : t - 1, s->d_L, B};
    if (t == 0 && s->vt_bf16) {  // the epilogue also writes V transposed for the tensor-core attention
      ra.vtpair_hi = s->vt_bf16 + (((long)s->cur_user * c.layers + l) * c.kv_heads) * D * s->pbmaps.pair_cap;
      ra.pair_cap = s->pbmaps.pair_cap;
    }
    FWD_TRY(gemm16(s, s->h, w.pqkv, nullptr, qkvd, w.bqkv, M, qkvd, H, EPI_ROPE, &ra));
    if (t == 0 && s->tc_prefill)
      FWD_TRY(attention_prefill_tc_bf16(s->pbmaps, s->cur_user, l, c.layers, s->q, s->attn, M, c.heads, c.kv_heads, D,
                                        cap, scale, s->d_status, st));
    else if (t == 0)
      FWD_TRY(attention_prefill(s->q, kp, vp, s->attn, nullptr, nullptr, M, cap, c.heads, c.kv_heads, D, scale, true,
                                st));
    else
      FWD_TRY(decode_attention(s, l, kp, vp, ks, vs, t, nullptr, nullptr, scale, du));
    FWD_TRY(gemm16(s, s->attn, w.po, s->x, H, nullptr, M, H, qd, EPI_RESID));
    FWD_TRY(rms_norm_rows_bf16(s->x, w.n_post, s->h, M, H, c.rms_eps, st));
    FWD_TRY(gemm16(s, s->h, w.pgu, s->act, I, nullptr, M, 2 * I, H, EPI_SWIGLU));
    FWD_TRY(gemm16(s, s->act, w.pd, s->x, H, nullptr, M, H, I, EPI_RESID));
  }
  if (t == 0) {  // the last position only
    const uint16_t* last = reinterpret_cast<const uint16_t*>(s->x) + (size_t)(M - 1) * H;
    FWD_TRY(rms_norm_rows_bf16(last, s->norm_final, s->h, 1, H, c.rms_eps, st));
    FWD_TRY(gemm16(s, s->h, s->lm_packed_bf, s->logits, V, nullptr, 1, V, H, EPI_STORE));
  } else {
    FWD_TRY(rms_norm_rows_bf16(s->x, s->norm_final, s->h, M, H, c.rms_eps, st));
    FWD_TRY(gemm16(s, s->h, s->lm_packed_bf, s->logits, V, nullptr, M, V, H, EPI_STORE, nullptr,
                   s->lse_tail ? s->lse : nullptr));
  }
  return cudaSuccess;
}

// t = 0: prefill of L rows (host L); t >= 1: decode step with beams rows.
static cudaError_t forward(rtr_session* s, int t) {
  if (s->bf16) return forward_bf16(s, t);
  const auto& c = s->cfg;
  const int H = c.hidden, V = c.vocab, I = c.intermediate, D = c.head_dim;
  const int qd = c.heads * D, kvd = c.kv_heads * D, qkvd = qkv_dim(c);
  const int B = beams_of(s), cap = c.max_prefix;
  // t = 0: user cur_user's prefill; t >= 1: one decode step of step_users users
  const int n = s->step_users, RB = B * s->max_users;
  const int M = t == 0 ? s->Ls[s->cur_user] : B * n;
  const long pre_off = t == 0 ? (long)s->cur_user * s->prefix_user : 0;
  const DecodeUsers du{n, s->prefix_user, (int)(sizeof(BeamState) / sizeof(int32_t))};
  const float scale = (float)std::pow((double)D, -0.5);
  cudaStream_t st = s->stream;
  const int32_t* ids = t == 0 ? s->d_ids : &s->beam->next_tok[0];
  const int id_rows = t == 0 ? 0 : B;  // decode: user m / B's beam m % B
  const long id_stride = (long)(sizeof(BeamState) / sizeof(int32_t));
  if (s->fold) {
    // RMSNorm folded into the GEMMs: the residual stream's producers write x, its
    // split and partial sums of squares; q/k/v, gate/up and the LM head scale rows
    const NormFold in{nullptr, s->ss, s->ss_ld, H / 128, H, c.rms_eps};
    const NormFold out{s->ss, nullptr, s->ss_ld, H / 128, H, c.rms_eps};
    FWD_TRY(embed_rows(ids, 1, M, s->embed, V, H, s->x, s->d_status, st, s->x_big, s->x_small, s->ss, s->ss_ld,
                       id_rows, id_stride, s->xfmt));
    for (int l = 0; l < c.layers; ++l) {
      const LayerW& w = s->layers[l];
      float* kp = s->kv_prefix + pre_off + (size_t)l * 2 * kvd * cap;
      float* vp = kp + (size_t)kvd * cap;
      float* ks = s->kv_suffix + (size_t)l * 2 * 4 * RB * kvd;
      float* vs = ks + (size_t)4 * RB * kvd;
      const size_t slot = t == 0 ? 0 : (size_t)(t - 1) * B * n * kvd;
      RopeArgs ra{s->rope_cos, s->rope_sin, s->rope_positions, c.heads, c.kv_heads, D, s->q,
                  t == 0 ? kp : ks + slot, t == 0 ? vp : vs + slot, cap, t == 0 ? -1 : t - 1, s->d_L, B};
      if (t == 0) set_pair_copies(s, ra, l);
      FWD_TRY(gemm(s, s->x, H, w.wqkv, s->qkv, qkvd, w.bqkv, M, qkvd, H, EPI_ROPE, &ra, &in));
      if (t == 0) {
        FWD_TRY(prefill_attention(s, l, kp, vp, M, scale));
      } else {
        FWD_TRY(decode_attention(s, l, kp, vp, ks, vs, t, s->attn_big, s->attn_small, scale, du));
      }
      FWD_TRY(gemm(s, s->attn, qd, w.wo, s->x, H, nullptr, M, H, qd, EPI_RESID, nullptr, &out));
      FWD_TRY(gemm(s, s->x, H, w.wgu, s->act, I, nullptr, M, 2 * I, H, EPI_SWIGLU, nullptr, &in));
      FWD_TRY(gemm(s, s->act, I, w.wd, s->x, H, nullptr, M, H, I, EPI_RESID, nullptr, &out));
    }
    if (t == 0) {  // the prefill's last row: explicit norm and the unfolded LM head (GEMV)
      FWD_TRY(rms_norm_rows(s->x + (size_t)(M - 1) * H, s->norm_final, s->h, nullptr, nullptr, 1, H, c.rms_eps, st));
      FWD_TRY(gemv_f32(s->h, s->lm_head, s->logits, V, H, st));
    } else {
      FWD_TRY(gemm(s, s->x, H, s->lm_head, s->logits, V, nullptr, M, V, H, EPI_STORE, nullptr, &in,
                   s->lse_tail ? s->lse : nullptr));
    }
    return cudaSuccess;
  }
  FWD_TRY(embed_rows(ids, 1, M, s->embed, V, H, s->x, s->d_status, st, nullptr, nullptr, nullptr, 0, id_rows,
                     id_stride));
  for (int l = 0; l < c.layers; ++l) {
    const LayerW& w = s->layers[l];
    float* kp = s->kv_prefix + pre_off + (size_t)l * 2 * kvd * cap;
    float* vp = kp + (size_t)kvd * cap;
    float* ks = s->kv_suffix + (size_t)l * 2 * 4 * RB * kvd;
    float* vs = ks + (size_t)4 * RB * kvd;
    FWD_TRY(rms_norm_rows(s->x, w.n_in, s->h, s->h_big, s->h_small, M, H, c.rms_eps, st, s->xfmt));
    const size_t slot = t == 0 ? 0 : (size_t)(t - 1) * B * n * kvd;
    if (s->use_tc) {
      // q/k/v projection with RoPE and the cache write fused into its epilogue
      RopeArgs ra{s->rope_cos, s->rope_sin, s->rope_positions, c.heads, c.kv_heads, D, s->q,
                  t == 0 ? kp : ks + slot, t == 0 ? vp : vs + slot, cap, t == 0 ? -1 : t - 1, s->d_L, B};
      if (t == 0) set_pair_copies(s, ra, l);
      FWD_TRY(gemm(s, s->h, H, w.wqkv, s->qkv, qkvd, w.bqkv, M, qkvd, H, EPI_ROPE, &ra));
    } else {
      FWD_TRY(gemm(s, s->h, H, w.wqkv, s->qkv, qkvd, w.bqkv, M, qkvd, H, EPI_BIAS));
      FWD_TRY(rope_kv(s->qkv, M, c.heads, c.kv_heads, D, s->rope_cos, s->rope_sin, s->rope_positions, s->q,
                      t == 0 ? kp : ks + slot, t == 0 ? vp : vs + slot, cap, t == 0 ? -1 : t - 1, s->d_L,
                      s->d_status, st));
    }
    if (t == 0) {
      FWD_TRY(prefill_attention(s, l, kp, vp, M, scale));
    } else {
      FWD_TRY(decode_attention(s, l, kp, vp, ks, vs, t, s->attn_big, s->attn_small, scale, du));
    }
    FWD_TRY(gemm(s, s->attn, qd, w.wo, s->x, H, nullptr, M, H, qd, EPI_RESID));
    FWD_TRY(rms_norm_rows(s->x, w.n_post, s->h, s->h_big, s->h_small, M, H, c.rms_eps, st, s->xfmt));
    FWD_TRY(gemm(s, s->h, H, w.wgu, s->act, I, nullptr, M, 2 * I, H, EPI_SWIGLU));
    FWD_TRY(gemm(s, s->act, I, w.wd, s->x, H, nullptr, M, H, I, EPI_RESID));
  }
  if (t == 0) {
    FWD_TRY(rms_norm_rows(s->x + (size_t)(M - 1) * H, s->norm_final, s->h, nullptr, nullptr, 1, H, c.rms_eps, st));
    FWD_TRY(gemv_f32(s->h, s->lm_head, s->logits, V, H, st));
  } else {
    FWD_TRY(rms_norm_rows(s->x, s->norm_final, s->h, s->h_big, s->h_small, M, H, c.rms_eps, st, s->xfmt));
    FWD_TRY(gemm(s, s->h, H, s->lm_head, s->logits, V, nullptr, M, V, H, EPI_STORE, nullptr, nullptr,
                 s->lse_tail ? s->lse : nullptr));
  }
  return cudaSuccess;
}

static cudaError_t decode_and_tail(rtr_session* s, int t) {
  FWD_TRY(forward(s, t));
  return beam_step(s->beam, s->logits, beams_of(s), s->cfg.vocab, beams_of(s), t, s->tb, s->d_status, s->stream,
                   s->step_users, s->lse_tail ? s->lse : nullptr);
}

static cudaError_t finalize_and_copy(rtr_session* s) {
  FWD_TRY(beam_finalize(s->beam, beams_of(s), s->dres, s->d_status, s->stream, s->step_users));
  return cudaMemcpyAsync(s->hres, s->dres, s->step_users * sizeof(DevResult), cudaMemcpyDeviceToHost, s->stream);
}

static int ready(rtr_session* s) {
  if (!s->weights_loaded) return fail(s, RTR_ERR_STATE, "weights not loaded");
  if (!s->tables_loaded) return fail(s, RTR_ERR_STATE, "constraint tables not loaded");
  return RTR_OK;
}


// Kernels one forward pass launches: embedding, per layer RMSNorm, q/k/v GEMM,
// RoPE + cache write (fused into the q/k/v GEMM on the tensor-core path),
// attention, o GEMM, RMSNorm, gate/up GEMM, down GEMM; then the final RMSNorm
// and the LM head.  With the norm fold the per-layer RMSNorms vanish and the
// decode step's final norm lives in the LM-head GEMM (the prefill keeps it for
// its one-row GEMV).  The step tail is 4 (max, two sums, beam selection).
static int64_t forward_kernels(const rtr_session* s, bool prefill) {
  if (s->fold) return 1 + 5 * (int64_t)s->cfg.layers + (prefill ? 2 : 1);
  return 1 + (s->use_tc ? 7 : 8) * (int64_t)s->cfg.layers + 2;
}
static constexpr int64_t kTailKernels = 4;   // step 0 (the prefill's GEMV LM head)
static int64_t decode_tail_kernels(const rtr_session* s) { return s->lse_tail ? 2 : kTailKernels; }

static int check_prompt(rtr_session* s, const int32_t* ids, int32_t L) {
  if (!ids) return fail(s, RTR_ERR_ARG, "null ids");
  if (L < 3 || L > s->cfg.max_prefix)
    return fail(s, RTR_ERR_ARG, "Expected one complete history within prefix capacity (3 <= L <= max_prefix)");
  return RTR_OK;
}

// Prefill of user u (its own prefix arena, length slot and beam state) and its
// step 0.  User 0 also clears the batch's status word.
static int stage_prefill(rtr_session* s, const int32_t* ids, int32_t L, int32_t on_device, int u = 0) {
  if (int r = check_prompt(s, ids, L)) return r;
  if (int r = ready(s)) return r;
  CUDA_TRY(s, cudaSetDevice(s->device));
  s->L = L;
  s->Ls[u] = L;
  s->cur_user = u;
  s->h_L[u] = L;
  CUDA_TRY(s, cudaMemcpyAsync(s->d_L + u, s->h_L + u, sizeof(int32_t), cudaMemcpyHostToDevice, s->stream));
  CUDA_TRY(s, cudaMemcpyAsync(s->d_ids, ids, (size_t)L * sizeof(int32_t),
                              on_device ? cudaMemcpyDeviceToDevice : cudaMemcpyHostToDevice, s->stream));
  if (u == 0) CUDA_TRY(s, cudaMemsetAsync(s->d_status, 0, sizeof(uint32_t), s->stream));
  CUDA_TRY(s, beam_reset(s->beam + u, s->d_ids, s->d_L + u, beams_of(s), s->stream));
  CUDA_TRY(s, forward(s, 0));
  CUDA_TRY(s, beam_step(s->beam + u, s->logits, 1, s->cfg.vocab, beams_of(s), 0, s->tb, s->d_status, s->stream));
  s->launches += 1 + forward_kernels(s, true) + kTailKernels;  // beam_reset, forward, step tail
  s->steps_done = 0;
  s->in_flight = false;
  return RTR_OK;
}

static std::string status_hex(uint32_t st) {
  char b[16];
  snprintf(b, sizeof b, "0x%x", st);
  return b;
}

static int check_result(rtr_session* s, const rtr_result* out, int u = 0) {
  const DevResult& r = s->hres[u];
  const uint32_t st = r.status;
  if (st & RTR_DEV_TIMEOUT) {
    // the aborted GEMMs keep their split-K tickets whole; re-arm them anyway so
    // no count left by an interrupted launch can reach the next request
    CUDA_TRY(s, cudaMemsetAsync(s->tickets, 0, kTickets * sizeof(int), s->stream));
    return fail(s, RTR_ERR_DEVICE, "a bounded pipeline wait ran out (status " + status_hex(st) + ")");
  }
  if (st & (RTR_DEV_BAD_TOKEN | RTR_DEV_BAD_PARENT | RTR_DEV_BAD_LENGTH | RTR_DEV_TOO_MANY_CAND | RTR_DEV_NAN_SCORE))
    return fail(s, RTR_ERR_DEVICE, "device bound check failed (status " + status_hex(st) + ")");
  if (st & RTR_DEV_NOT_STOPPED)
    return fail(s, RTR_ERR_DEVICE, "beam search would continue after 5 steps (catalog grammar is not 3 SID tokens + newline + EOS)");
  if (st & RTR_DEV_STOPPED_EARLY)
    return fail(s, RTR_ERR_DEVICE, "beam search stopped before 5 steps");
  const int B = beams_of(s);
  if (out) {
    if (out->token_ids) memcpy(out->token_ids, r.token_ids, sizeof(int32_t) * B * NSTEPS);
    if (out->beam_indices) memcpy(out->beam_indices, r.beam_indices, sizeof(int32_t) * B * NSTEPS);
    if (out->sequence_logp) memcpy(out->sequence_logp, r.sequence_logp, sizeof(float) * B);
    if (out->transition_logp) memcpy(out->transition_logp, r.transition_logp, sizeof(float) * B * NSTEPS);
  }
  s->err = (st & RTR_DEV_FEW_FINITE) ? "warning: fewer finite candidates than beams at some step" : "";
  return RTR_OK;
}

extern "C" {

int rtr_prefill(rtr_session* s, const int32_t* ids, int32_t L, int32_t ids_on_device) {
  if (!s) return RTR_ERR_ARG;
  if (s->in_flight) return fail(s, RTR_ERR_STATE, "request in flight");
  s->step_users = 1;
  return stage_prefill(s, ids, L, ids_on_device);
}

int rtr_decode_step(rtr_session* s, int32_t t) {
  if (!s) return RTR_ERR_ARG;
  if (t < 1 || t >= NSTEPS) return fail(s, RTR_ERR_ARG, "decode step must be in 1..4");
  if (s->steps_done != t - 1) return fail(s, RTR_ERR_STATE, "decode steps must follow prefill in order");
  CUDA_TRY(s, cudaSetDevice(s->device));
  CUDA_TRY(s, decode_and_tail(s, t));
  s->launches += forward_kernels(s, false) + decode_tail_kernels(s);
  s->steps_done = t;
  return RTR_OK;
}

int rtr_read_results(rtr_session* s, const rtr_result* out) {
  if (!s) return RTR_ERR_ARG;
  if (s->steps_done != NSTEPS - 1) return fail(s, RTR_ERR_STATE, "all four decode steps must run first");
  CUDA_TRY(s, cudaSetDevice(s->device));
  CUDA_TRY(s, finalize_and_copy(s));
  s->launches += 1;
  CUDA_TRY(s, cudaStreamSynchronize(s->stream));
  return check_result(s, out);
}

// One request of n users: each user's prefill (and step 0) runs eagerly, then
// one captured graph runs decode steps 1-4 for all n users together (every
// projection GEMM at n * beams rows) and copies the results out.
static int launch_batch(rtr_session* s, const int32_t* const* ids, const int32_t* L, int32_t n, int32_t ids_on_device) {
  if (!ids || !L) return fail(s, RTR_ERR_ARG, "null ids or lengths");
  if (n < 1 || n > s->max_users) return fail(s, RTR_ERR_ARG, "user count must be in [1, max_users]");
  for (int u = 0; u < n; ++u)
    if (int r = check_prompt(s, ids[u], L[u])) return r;
  if (int r = ready(s)) return r;
  CUDA_TRY(s, cudaSetDevice(s->device));
  s->step_users = n;
  if (!s->graphs[n]) {
    cudaGraph_t g = nullptr;
    CUDA_TRY(s, cudaStreamBeginCapture(s->stream, cudaStreamCaptureModeThreadLocal));
    cudaError_t e = cudaSuccess;
    for (int t = 1; t < NSTEPS && e == cudaSuccess; ++t) e = decode_and_tail(s, t);
    if (e == cudaSuccess) e = finalize_and_copy(s);
    cudaError_t e2 = cudaStreamEndCapture(s->stream, &g);
    if (e != cudaSuccess || e2 != cudaSuccess) {
      if (g) cudaGraphDestroy(g);
      return fail(s, RTR_ERR_CUDA, std::string("decode graph capture: ") +
                                       cudaGetErrorString(e != cudaSuccess ? e : e2));
    }
    size_t nodes_n = 0;
    cudaGraphGetNodes(g, nullptr, &nodes_n);
    std::vector<cudaGraphNode_t> nodes(nodes_n);
    cudaGraphGetNodes(g, nodes.data(), &nodes_n);
    s->graph_kernels = 0;
    for (auto node : nodes) {
      cudaGraphNodeType ty;
      if (cudaGraphNodeGetType(node, &ty) == cudaSuccess && ty == cudaGraphNodeTypeKernel) ++s->graph_kernels;
    }
    e = cudaGraphInstantiate(&s->graphs[n], g, 0);
    cudaGraphDestroy(g);
    if (e != cudaSuccess) {
      s->graphs[n] = nullptr;
      return fail(s, RTR_ERR_CUDA, std::string("graph instantiate: ") + cudaGetErrorString(e));
    }
  }
  // Device ids may be queued behind a request in flight (stream order keeps
  // them apart); host ids reuse the pinned staging buffer, so wait first.
  if (s->in_flight && !ids_on_device) CUDA_TRY(s, cudaStreamSynchronize(s->stream));
  for (int u = 0; u < n; ++u) {
    const int32_t* src = ids[u];
    if (!ids_on_device) {
      // stage the prompt through pinned memory so the copy is asynchronous
      int32_t* pin = s->h_ids + (size_t)u * s->cfg.max_prefix;
      memcpy(pin, ids[u], (size_t)L[u] * sizeof(int32_t));
      src = pin;
    }
    if (int r = stage_prefill(s, src, L[u], ids_on_device, u)) return r;
  }
  CUDA_TRY(s, cudaGraphLaunch(s->graphs[n], s->stream));
  s->launches += s->graph_kernels;
  s->requests += n;
  s->steps_done = NSTEPS - 1;
  s->in_flight = true;
  return RTR_OK;
}

int rtr_launch(rtr_session* s, const int32_t* ids, int32_t L, int32_t ids_on_device) {
  if (!s) return RTR_ERR_ARG;
  return launch_batch(s, &ids, &L, 1, ids_on_device);
}

int rtr_launch_batch(rtr_session* s, const int32_t* const* ids, const int32_t* L, int32_t n_users,
                     int32_t ids_on_device) {
  if (!s) return RTR_ERR_ARG;
  return launch_batch(s, ids, L, n_users, ids_on_device);
}

int rtr_wait_batch(rtr_session* s, const rtr_result* out) {
  if (!s) return RTR_ERR_ARG;
  if (!s->in_flight) return fail(s, RTR_ERR_STATE, "no request in flight");
  CUDA_TRY(s, cudaSetDevice(s->device));
  s->in_flight = false;
  CUDA_TRY(s, cudaStreamSynchronize(s->stream));
  for (int u = 0; u < s->step_users; ++u)
    if (int r = check_result(s, out ? out + u : nullptr, u)) return r;
  return RTR_OK;
}

int rtr_wait(rtr_session* s, const rtr_result* out) {
  if (!s) return RTR_ERR_ARG;
  if (s->in_flight && s->step_users != 1) return fail(s, RTR_ERR_STATE, "a batch is in flight: use rtr_wait_batch");
  return rtr_wait_batch(s, out);
}

int rtr_generate(rtr_session* s, const int32_t* ids_host, int32_t L, const rtr_result* out) {
  if (int r = rtr_launch(s, ids_host, L, 0)) return r;
  return rtr_wait(s, out);
}

int rtr_generate_batch(rtr_session* s, const int32_t* const* ids_host, const int32_t* L, int32_t n_users,
                       const rtr_result* out) {
  if (int r = rtr_launch_batch(s, ids_host, L, n_users, 0)) return r;
  return rtr_wait_batch(s, out);
}

int rtr_get_report(const rtr_session* s, rtr_report* out) {
  if (!s || !out) return RTR_ERR_ARG;
  const auto& c = s->cfg;
  const int64_t kvd = (int64_t)c.kv_heads * c.head_dim, B = c.num_beams;
  memset(out, 0, sizeof(*out));
  out->requests = s->requests;
  out->kernel_launches = s->launches;
  // beam_reset + NSTEPS x (forward + step tail) + beam_finalize
  out->launches_per_request =
      1 + forward_kernels(s, true) + (NSTEPS - 1) * forward_kernels(s, false) + kTailKernels +
      (NSTEPS - 1) * decode_tail_kernels(s) + 1;
  out->graph_kernel_nodes = s->graph_kernels;
  out->prefix_bytes_written = (int64_t)c.layers * 2 * kvd * s->L * (int64_t)sizeof(float);
  out->prefix_bytes_reordered = 0;
  out->suffix_bytes_written = (int64_t)c.layers * 2 * kvd * B * (NSTEPS - 1) * (int64_t)sizeof(float);
  out->suffix_bytes_gathered = 0;
  out->weight_bytes = s->weight_bytes;
  out->device_bytes = s->device_bytes;
  out->h2d_bytes_per_request = (int64_t)s->L * 4 + 4;
  out->d2h_bytes_per_request = (int64_t)sizeof(DevResult);
  out->tensor_core_gemm = s->use_tc ? (s->xfmt == SPLIT_F16 ? 2 : 1) : 0;
  out->norm_fold = s->fold ? 1 : 0;
  out->decode_attention = s->tc_attn || s->tc_attn_bf16 ? 1 : s->folded_attn ? 2 : 0;
  out->prefill_attention = s->tc_prefill ? 1 : 0;
  return RTR_OK;
}

int rtr_profile_gemms(rtr_session* s, int32_t M, int32_t reps, float* ms_per_pass) {
  if (!s || !ms_per_pass || reps < 1) return RTR_ERR_ARG;
  const int rows = s->cfg.num_beams * s->max_users;
  if (M < 1 || M > (s->cfg.max_prefix > rows ? s->cfg.max_prefix : rows))
    return fail(s, RTR_ERR_ARG, "M outside the activation buffers");
  if (s->in_flight) return fail(s, RTR_ERR_STATE, "request in flight");
  if (!s->weights_loaded) return fail(s, RTR_ERR_STATE, "weights not loaded");
  CUDA_TRY(s, cudaSetDevice(s->device));
  const auto& c = s->cfg;
  const int H = c.hidden, I = c.intermediate, qd = c.heads * c.head_dim, qkvd = qkv_dim(c);
  cudaEvent_t a, b;
  CUDA_TRY(s, cudaEventCreate(&a));
  CUDA_TRY(s, cudaEventCreate(&b));
  auto pass = [&]() -> cudaError_t {
    if (s->bf16) {
      for (int l = 0; l < c.layers; ++l) {
        const LayerW& w = s->layers[l];
        FWD_TRY(gemm16(s, s->h, w.pqkv, s->qkv, qkvd, w.bqkv, M, qkvd, H, EPI_BIAS));
        FWD_TRY(gemm16(s, s->attn, w.po, s->x, H, nullptr, M, H, qd, EPI_STORE));
        FWD_TRY(gemm16(s, s->h, w.pgu, s->act, I, nullptr, M, 2 * I, H, EPI_SWIGLU));
        FWD_TRY(gemm16(s, s->act, w.pd, s->x, H, nullptr, M, H, I, EPI_STORE));
      }
      return gemm16(s, s->h, s->lm_packed_bf, s->logits, c.vocab, nullptr, M < c.num_beams ? M : c.num_beams,
                    c.vocab, H, EPI_STORE);
    }
    for (int l = 0; l < c.layers; ++l) {
      const LayerW& w = s->layers[l];
      FWD_TRY(gemm(s, s->h, H, w.wqkv, s->qkv, qkvd, w.bqkv, M, qkvd, H, EPI_BIAS));
      FWD_TRY(gemm(s, s->attn, qd, w.wo, s->x, H, nullptr, M, H, qd, EPI_STORE));
      FWD_TRY(gemm(s, s->h, H, w.wgu, s->act, I, nullptr, M, 2 * I, H, EPI_SWIGLU));
      FWD_TRY(gemm(s, s->act, I, w.wd, s->x, H, nullptr, M, H, I, EPI_STORE));
    }
    return gemm(s, s->h, H, s->lm_head, s->logits, c.vocab, nullptr, M < c.num_beams ? M : c.num_beams,
                c.vocab, H, EPI_STORE);
  };
  cudaError_t e = pass();  // warm-up
  if (e == cudaSuccess) e = cudaEventRecord(a, s->stream);
  for (int r = 0; r < reps && e == cudaSuccess; ++r) e = pass();
  if (e == cudaSuccess) e = cudaEventRecord(b, s->stream);
  if (e == cudaSuccess) e = cudaEventSynchronize(b);
  float ms = 0.f;
  if (e == cudaSuccess) e = cudaEventElapsedTime(&ms, a, b);
  cudaEventDestroy(a);
  cudaEventDestroy(b);
  if (e != cudaSuccess) return fail(s, RTR_ERR_CUDA, std::string("profile: ") + cudaGetErrorString(e));
  *ms_per_pass = ms / reps;
  return RTR_OK;
}

int rtr_step_scores(rtr_session* s, int32_t t, float* out_dev) {
  if (!s || !out_dev) return RTR_ERR_ARG;
  if (t < 0 || t >= NSTEPS) return fail(s, RTR_ERR_ARG, "step must be in 0..4");
  if (s->steps_done < t) return fail(s, RTR_ERR_STATE, "step has not run");
  CUDA_TRY(s, cudaSetDevice(s->device));
  CUDA_TRY(s, beam_dense_scores(s->beam, t, beams_of(s), s->cfg.vocab, out_dev, s->stream));
  CUDA_TRY(s, cudaStreamSynchronize(s->stream));
  return RTR_OK;
}

int rtr_lookup_width(const rtr_session* s, int32_t step, int32_t* width) {
  if (!s || !width || !s->tables_loaded || step < 0) return RTR_ERR_ARG;
  *width = lookup_width(s->tb, step);
  return RTR_OK;
}

int rtr_constraint_lookup(rtr_session* s, int32_t step, const int64_t* input_ids_dev, int32_t rows,
                          int32_t cols, int32_t* out_dev) {
  if (!s || !input_ids_dev || !out_dev || rows < 1) return RTR_ERR_ARG;
  if (!s->tables_loaded) return fail(s, RTR_ERR_STATE, "constraint tables not loaded");
  if (step < 0) return fail(s, RTR_ERR_ARG, "negative step");
  const int need = (step == 0 || step == 3) ? 3 : (step < 3 ? step : 0);
  if (cols < need) return fail(s, RTR_ERR_ARG, "input_ids shorter than the step's prefix");
  CUDA_TRY(s, cudaSetDevice(s->device));
  CUDA_TRY(s, constraint_lookup(s->tb, step, input_ids_dev, rows, cols, out_dev, s->stream));
  CUDA_TRY(s, cudaStreamSynchronize(s->stream));
  return RTR_OK;
}

int rtr_constraint_process(rtr_session* s, int32_t step, const int64_t* input_ids_dev, int32_t rows,
                           int32_t cols, const float* scores_dev, float* out_dev) {
  if (!s || !input_ids_dev || !scores_dev || !out_dev || rows < 1) return RTR_ERR_ARG;
  if (!s->tables_loaded) return fail(s, RTR_ERR_STATE, "constraint tables not loaded");
  if (scores_dev == out_dev) return fail(s, RTR_ERR_ARG, "output aliases the scores");
  if (step < 0) return fail(s, RTR_ERR_ARG, "negative step");
  const int need = (step == 0 || step == 3) ? 3 : (step < 3 ? step : 0);
  if (cols < need) return fail(s, RTR_ERR_ARG, "input_ids shorter than the step's prefix");
  if (rows > PROC_MAX_ROWS) return fail(s, RTR_ERR_ARG, "at most 4096 rows per call");
  CUDA_TRY(s, cudaSetDevice(s->device));
  CUDA_TRY(s, constraint_process(s->tb, step, input_ids_dev, rows, cols, scores_dev, out_dev, s->cfg.vocab,
                                 s->proc_scratch, s->stream));
  CUDA_TRY(s, cudaStreamSynchronize(s->stream));
  return RTR_OK;
}

int rtr_constraint_process_static(rtr_session* s, int32_t step, const int64_t* input_ids_dev, int32_t rows,
                                  int32_t cols, const float* scores_dev, float* out_dev) {
  if (!s || !input_ids_dev || !scores_dev || !out_dev || rows < 1) return RTR_ERR_ARG;
  if (!s->tables_loaded) return fail(s, RTR_ERR_STATE, "constraint tables not loaded");
  if (scores_dev == out_dev) return fail(s, RTR_ERR_ARG, "output aliases the scores");
  if (step < 0) return fail(s, RTR_ERR_ARG, "negative step");
  const int need = (step == 0 || step == 3) ? 3 : (step < 3 ? step : 0);
  if (cols < need) return fail(s, RTR_ERR_ARG, "input_ids shorter than the step's prefix");
  if (rows > STATIC_PROC_MAX_ROWS)
    return fail(s, RTR_ERR_ARG, "rtr_constraint_process_static serves at most 256 rows (its static scratch size)");
  CUDA_TRY(s, cudaSetDevice(s->device));
  CUDA_TRY(s, constraint_process_static(s->tb, step, input_ids_dev, rows, cols, scores_dev, out_dev, s->cfg.vocab,
                                        s->stream));
  CUDA_TRY(s, cudaStreamSynchronize(s->stream));
  return RTR_OK;
}

int rtr_synth_fill_host(float* dst, int64_t n, uint64_t seed, uint64_t tid, float scale, float offset) {
  if (!dst || n < 0) return RTR_ERR_ARG;
  synth_fill_host(dst, n, seed, tid, scale, offset);
  return RTR_OK;
}

int rtr_synth_fill_device(float* dst_dev, int64_t n, uint64_t seed, uint64_t tid, float scale, float offset,
                          void* stream) {
  if (!dst_dev || n < 0) return RTR_ERR_ARG;
  cudaError_t e = synth_fill_device(dst_dev, n, seed, tid, scale, offset, static_cast<cudaStream_t>(stream));
  if (e == cudaSuccess) e = cudaStreamSynchronize(static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return fail(nullptr, RTR_ERR_CUDA, cudaGetErrorString(e));
  return RTR_OK;
}

}  // extern "C"
