// The fused step tail of the constrained beam search, on device.
//
// One beam-search iteration of transformers' GenerationMixin._beam_search
// (generation/utils.py:3252-3352) with the reference's processor
// GpuSidConstrainedLogitsProcessor (rapidtinyrec/gpu_constraints.py:90-101):
//
//   lp1 = log_softmax(float(logits))            three passes over the vocabulary,
//   lp2 = log_softmax(lp1)                      split over TAIL_SPLITS CTAs/row
//   scores = lp2 + mask(lookup(step, ids))      only allowed columns are finite
//   acc = scores + running_scores               candidates = allowed columns
//   topk(acc, 2*beams) -> EOS hits -> running topk(beams) -> finished merge
//   -> parents (cache reorder) -> early-stop heuristic
//
// Only the allowed columns can be finite, so the candidate set is
// beams x width (<= 64 x 256) instead of beams x vocab; a single CTA radix-
// selects the top 2*beams 64-bit keys (order-preserving score bits, then the
// complemented flat index, so equal scores rank the lower flat index first).
// log_softmax keeps torch's CPU form (x - max) - log(sum exp(x - max)); the
// second pass's max is exactly -log(sum) of the first.
#include <math.h>

#include <mutex>

#include "common.cuh"
#include "engine.h"

namespace rtr {

constexpr int TAIL_THREADS = 256;
constexpr int SEL_THREADS = 1024;
constexpr int MAX_CAND = MAX_BEAMS * MAX_WIDTH;

// Deterministic block reductions (fixed shuffle tree, warps summed in order).
__device__ float block_sum(float v, float* red) {
  v = warp_sum(v);
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  __syncthreads();
  if (l == 0) red[w] = v;
  __syncthreads();
  float r = 0.f;
  if (threadIdx.x == 0) {
    for (int i = 0; i < (int)(blockDim.x >> 5); ++i) r += red[i];
    red[32] = r;
  }
  __syncthreads();
  return red[32];
}

__device__ float block_max(float v, float* red) {
  v = warp_max(v);
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  __syncthreads();
  if (l == 0) red[w] = v;
  __syncthreads();
  if (threadIdx.x == 0) {
    float r = -INFINITY;
    for (int i = 0; i < (int)(blockDim.x >> 5); ++i) r = fmaxf(r, red[i]);
    red[32] = r;
  }
  __syncthreads();
  return red[32];
}

// ---------------------------------------------------------- SID lookup
// Row descriptor of GpuSidConstraintTables.lookup (gpu_constraints.py:69-87).
struct LookupRow {
  int kind;   // 0: first tokens, 1: one token broadcast, 2: table1 row, 3: table2 row
  int token;  // kind 1
  long index; // kinds 2/3
};

__device__ __forceinline__ bool sid_index(const DevTables& tb, const long* tok, int n, long* index) {
  bool in_range = true;
  long idx = 0, stride = 1, limit = 1;
  for (int j = n - 1; j >= 0; --j) {
    const long digit = tok[j] - tb.offsets[j];
    in_range = in_range && digit >= 0 && digit < tb.sizes[j];
    idx += digit * stride;
    stride *= tb.sizes[j];
  }
  for (int j = 0; j < n; ++j) limit *= tb.sizes[j];
  idx = idx < 0 ? 0 : (idx > limit - 1 ? limit - 1 : idx);
  *index = idx;
  return in_range;
}

// tok[0..n) are the last n tokens of the row (oldest first); n = 3 at steps 0/3.
__device__ LookupRow lookup_row(const DevTables& tb, int step, const long* tok) {
  LookupRow r{1, tb.eos, 0};
  if (step == 1 || step == 2) {
    long idx;
    if (sid_index(tb, tok, step, &idx)) { r.kind = step + 1; r.index = idx; }
  } else if (step == 0 || step == 3) {
    long idx;
    const bool in_range = sid_index(tb, tok, 3, &idx);
    r.token = (in_range && tb.valid[idx]) ? tb.newline : tb.eos;
    if (tok[0] == tb.root[0] && tok[1] == tb.root[1] && tok[2] == tb.root[2]) r.kind = 0;
  }
  return r;
}

__device__ __forceinline__ int lookup_col(const DevTables& tb, const LookupRow& r, int j) {
  switch (r.kind) {
    case 0: return tb.first_tokens[j];
    case 2: return tb.table1[r.index * tb.width1 + j];
    case 3: return tb.table2[r.index * tb.width2 + j];
    default: return r.token;
  }
}

__host__ __device__ int lookup_width_of(const DevTables& tb, int step) {
  if (step == 0 || step == 3) return tb.n_first;
  if (step == 1) return tb.width1;
  if (step == 2) return tb.width2;
  return 1;
}

int lookup_width(const DevTables& tb, int step) { return lookup_width_of(tb, step); }

// -------------------------------------------------- vocabulary passes
// f(x[i]) for the thread's elements i = lo + tid + k * TAIL_THREADS of a row
// slice, in that order (the order of the plain loop, so the same bits), TB at
// a time with every load of a batch issued before the first is used: a slice
// of ~9,500 columns costs three L2 round trips instead of ten.
template <typename F>
RTR_DEVICE void for_slice(const float* __restrict__ x, long lo, long hi, F f) {
  constexpr int TB = 16;
  for (long i0 = lo + threadIdx.x; i0 < hi; i0 += (long)TB * TAIL_THREADS) {
    float v[TB];
#pragma unroll
    for (int k = 0; k < TB; ++k) {
      const long i = i0 + (long)k * TAIL_THREADS;
      v[k] = i < hi ? x[i] : 0.f;
    }
#pragma unroll
    for (int k = 0; k < TB; ++k)
      if (i0 + (long)k * TAIL_THREADS < hi) f(v[k]);
  }
}

__global__ void tail_max_kernel(const float* __restrict__ logits, int vocab, BeamState* st, int rows_per_user) {
  pdl_launch_dependents();
  pdl_wait();
  __shared__ float red[33];
  st += blockIdx.x / rows_per_user;  // batched decode: each user's rows feed its own state
  const int grow = blockIdx.x, row = blockIdx.x % rows_per_user, sp = blockIdx.y;
  const long lo = (long)vocab * sp / TAIL_SPLITS, hi = (long)vocab * (sp + 1) / TAIL_SPLITS;
  const float* x = logits + (long)grow * vocab;
  float m = -INFINITY;
  for_slice(x, lo, hi, [&](float v) { m = fmaxf(m, v); });
  m = block_max(m, red);
  if (threadIdx.x == 0) st->part[row][sp][0] = m;
}

__device__ __forceinline__ float row_max(const BeamState* st, int row) {
  float m = -INFINITY;
  for (int s = 0; s < TAIL_SPLITS; ++s) m = fmaxf(m, st->part[row][s][0]);
  return m;
}

__global__ void tail_sum1_kernel(const float* __restrict__ logits, int vocab, BeamState* st, int rows_per_user) {
  pdl_launch_dependents();
  pdl_wait();
  __shared__ float red[33];
  st += blockIdx.x / rows_per_user;  // batched decode: each user's rows feed its own state
  const int grow = blockIdx.x, row = blockIdx.x % rows_per_user, sp = blockIdx.y;
  const long lo = (long)vocab * sp / TAIL_SPLITS, hi = (long)vocab * (sp + 1) / TAIL_SPLITS;
  const float* x = logits + (long)grow * vocab;
  const float m = row_max(st, row);
  float s = 0.f;
  for_slice(x, lo, hi, [&](float v) { s += expf(v - m); });
  s = block_sum(s, red);
  if (threadIdx.x == 0) st->part[row][sp][1] = s;
}

__global__ void tail_sum2_kernel(const float* __restrict__ logits, int vocab, BeamState* st, int rows_per_user) {
  pdl_launch_dependents();
  pdl_wait();
  __shared__ float red[33];
  st += blockIdx.x / rows_per_user;  // batched decode: each user's rows feed its own state
  const int grow = blockIdx.x, row = blockIdx.x % rows_per_user, sp = blockIdx.y;
  const long lo = (long)vocab * sp / TAIL_SPLITS, hi = (long)vocab * (sp + 1) / TAIL_SPLITS;
  const float* x = logits + (long)grow * vocab;
  const float m = row_max(st, row);
  float s1 = 0.f;
  for (int k = 0; k < TAIL_SPLITS; ++k) s1 += st->part[row][k][1];
  const float L1 = logf(s1);
  const float m2 = (m - m) - L1;  // max of lp1, reached at the arg-max column
  float s = 0.f;
  for_slice(x, lo, hi, [&](float v) { s += expf(((v - m) - L1) - m2); });
  s = block_sum(s, red);
  if (threadIdx.x == 0) {
    st->part[row][sp][2] = s;
    if (sp == 0) { st->row_stats[row][0] = m; st->row_stats[row][1] = L1; st->row_stats[row][2] = m2; }
  }
}

// The second log-softmax pass when the LM head left per-tile (max, sum exp)
// partials: every CTA of a row first folds the row's partials in tile order
// into the row max m and the first sum s1 = sum_t s_t exp(m_t - m) (the same
// bits in each of the row's CTAs), then sums its slice of the second pass.
__global__ void tail_lse_sum2_kernel(const float* __restrict__ logits, int vocab, BeamState* st, int rows_per_user,
                                     const float2* __restrict__ lse) {
  pdl_launch_dependents();
  pdl_wait();
  __shared__ float red[33];
  st += blockIdx.x / rows_per_user;  // batched decode: each user's rows feed its own state
  const int grow = blockIdx.x, row = blockIdx.x % rows_per_user, sp = blockIdx.y;
  const int ntiles = (vocab + 127) / 128;
  const float2* part = lse + (long)grow * ntiles;
  // the thread's partials are loaded once, all in flight, and kept for both folds
  constexpr int PB = 8;  // ntiles <= PB * TAIL_THREADS (vocab <= 262,144)
  float2 pv[PB];
#pragma unroll
  for (int k = 0; k < PB; ++k) {
    const int t = threadIdx.x + k * TAIL_THREADS;
    pv[k] = t < ntiles ? part[t] : make_float2(-INFINITY, 0.f);
  }
  float m = -INFINITY;
#pragma unroll
  for (int k = 0; k < PB; ++k)
    if (threadIdx.x + k * TAIL_THREADS < ntiles) m = fmaxf(m, pv[k].x);
  m = block_max(m, red);
  float s1 = 0.f;
#pragma unroll
  for (int k = 0; k < PB; ++k)
    if (threadIdx.x + k * TAIL_THREADS < ntiles) s1 += pv[k].y * expf(pv[k].x - m);
  s1 = block_sum(s1, red);
  const long lo = (long)vocab * sp / TAIL_SPLITS, hi = (long)vocab * (sp + 1) / TAIL_SPLITS;
  const float* x = logits + (long)grow * vocab;
  const float L1 = logf(s1);
  const float m2 = (m - m) - L1;  // max of lp1, reached at the arg-max column
  float s = 0.f;
  for_slice(x, lo, hi, [&](float v) { s += expf(((v - m) - L1) - m2); });
  s = block_sum(s, red);
  if (threadIdx.x == 0) {
    st->part[row][sp][2] = s;
    if (sp == 0) { st->row_stats[row][0] = m; st->row_stats[row][1] = L1; st->row_stats[row][2] = m2; }
  }
}

// ---------------------------------------------------- select + update
__device__ __forceinline__ uint64_t cand_key(float acc, uint32_t flat) {
  return ((uint64_t)float_key(acc) << 32) | (uint64_t)(~flat);
}

struct SelShared {
  float stats[MAX_BEAMS][4];
  int32_t o_tok[MAX_BEAMS][NSTEPS], o_par[MAX_BEAMS][NSTEPS], o_anc[MAX_BEAMS][4];
  float o_score[MAX_BEAMS];
  int32_t f_tok[MAX_BEAMS][NSTEPS], f_par[MAX_BEAMS][NSTEPS], f_done[MAX_BEAMS];
  float f_score[MAX_BEAMS];
  LookupRow rows[MAX_BEAMS];
  int32_t col0[MAX_BEAMS];
  uint64_t top[2 * MAX_BEAMS];
  uint64_t sorted[2 * MAX_BEAMS];
  float c_score[2 * MAX_BEAMS], c_run[2 * MAX_BEAMS], c_fin[3 * MAX_BEAMS];
  int32_t c_beam[2 * MAX_BEAMS], c_tok[2 * MAX_BEAMS], c_hit[2 * MAX_BEAMS];
  int32_t n_run[MAX_BEAMS], n_fin[MAX_BEAMS];
  float nf_score[MAX_BEAMS];   // the new finished set, for the stop test
  int32_t nf_done[MAX_BEAMS];
  unsigned hist[256];
  unsigned char fmark[2 * MAX_BEAMS + MAX_WIDTH];  // row 0's allowed columns below K + width
  uint64_t prefix, mask;
  int krem, done, counter, finite;
  float red[33];
};

__global__ void __launch_bounds__(SEL_THREADS) beam_select_kernel(BeamState* st, const float* __restrict__ logits,
                                                                 int rows, int vocab, int beams, int step,
                                                                 DevTables tb, uint32_t* status) {
  pdl_launch_dependents();
  pdl_wait();
  extern __shared__ uint64_t cand[];
  __shared__ SelShared sh;
  st += blockIdx.x;  // batched decode: one block per user
  logits += (long)blockIdx.x * rows * vocab;
  const int tid = threadIdx.x, nt = blockDim.x;
  const int K = 2 * beams;
  const int width = lookup_width_of(tb, step);
  const int nc = beams * width;

  // 1. row statistics and a snapshot of the previous state
  if (tid < rows) {
    float s2 = 0.f;
    for (int k = 0; k < TAIL_SPLITS; ++k) s2 += st->part[tid][k][2];
    sh.stats[tid][0] = st->row_stats[tid][0];
    sh.stats[tid][1] = st->row_stats[tid][1];
    sh.stats[tid][2] = st->row_stats[tid][2];
    sh.stats[tid][3] = logf(s2);
    st->row_stats[tid][3] = sh.stats[tid][3];
  }
  for (int i = tid; i < beams * NSTEPS; i += nt) {
    const int b = i / NSTEPS, t = i % NSTEPS;
    sh.o_tok[b][t] = st->run_tok[b][t]; sh.o_par[b][t] = st->run_par[b][t];
    sh.f_tok[b][t] = st->fin_tok[b][t]; sh.f_par[b][t] = st->fin_par[b][t];
  }
  for (int b = tid; b < beams; b += nt) {
    sh.o_score[b] = st->run_score[b];
    sh.f_score[b] = st->fin_score[b];
    sh.f_done[b] = st->fin_done[b];
    for (int s = 0; s < 4; ++s) sh.o_anc[b][s] = st->anc[b][s];
    // lookup prefix: the last tokens of the running sequence
    long tok[3];
    if (step == 0) {
      for (int j = 0; j < 3; ++j) tok[j] = st->prompt_tail[j];
    } else if (step < 4) {
      const int n = step == 3 ? 3 : step;
      for (int j = 0; j < n; ++j) tok[j] = st->run_tok[b][step - n + j];
    }
    sh.rows[b] = lookup_row(tb, step, tok);
    sh.col0[b] = lookup_col(tb, sh.rows[b], 0);
  }
  if (tid == 0) { sh.finite = 0; st->width[step] = width; st->same_rows[step] = rows == 1; }
  __syncthreads();

  // 2. candidates: processed score at every allowed column
  int finite = 0;
  for (int i = tid; i < nc; i += nt) {
    const int b = i / width, j = i - b * width;
    int col = lookup_col(tb, sh.rows[b], j);
    if (col < 0 || col >= vocab) { atomicOr(status, RTR_DEV_BAD_TOKEN); col = 0; }
    const int r = rows == 1 ? 0 : b;
    const float x = logits[(long)r * vocab + col];
    const float lp1 = (x - sh.stats[r][0]) - sh.stats[r][1];
    const float v = (lp1 - sh.stats[r][2]) - sh.stats[r][3];
    st->cols[step][b][j] = col;
    st->vals[step][b][j] = v;
    float acc = v + sh.o_score[b];
    if (acc != acc) {  // NaN would break the rank permutation below
      atomicOr(status, RTR_DEV_NAN_SCORE);
      acc = -INFINITY;
    }
    const bool dup = j > 0 && col == sh.col0[b];
    uint64_t key = 0;
    if (!dup) {
      key = cand_key(acc, (uint32_t)(b * vocab + col));
      if (acc > -INFINITY) ++finite;
    }
    cand[i] = key;
  }
  finite = (int)block_sum((float)finite, sh.red);
  const int kk = finite < K ? finite : K;
  if (tid == 0) {
    if (finite < beams) atomicOr(status, RTR_DEV_FEW_FINITE);
    sh.prefix = 0; sh.mask = 0; sh.krem = kk; sh.done = kk == 0; sh.counter = 0;
  }
  __syncthreads();

  // 3. radix select of the kk largest keys (8-bit digits, MSB first)
  for (int pass = 0; pass < 8 && !sh.done; ++pass) {
    const int shift = 56 - 8 * pass;
    for (int i = tid; i < 256; i += nt) sh.hist[i] = 0;
    __syncthreads();
    const uint64_t pf = sh.prefix, mk = sh.mask;
    for (int i = tid; i < nc; i += nt) {
      const uint64_t k = cand[i];
      if ((k & mk) == pf) atomicAdd(&sh.hist[(k >> shift) & 255], 1u);
    }
    __syncthreads();
    if (tid < 32) {
      // the digit holding the krem-th largest key: the highest d whose bins
      // 255 .. d hold at least krem keys (bin 0 at the latest).  Lane l sums
      // bins 255 - 8 l .. 248 - 8 l, a warp scan orders the lanes, and the
      // first lane that reaches krem walks its own eight bins.
      const int lane = tid;
      const unsigned krem = (unsigned)sh.krem;
      unsigned c[8], tot = 0;
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        c[e] = sh.hist[255 - 8 * lane - e];
        tot += c[e];
      }
      unsigned incl = tot;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const unsigned v = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += v;
      }
      const unsigned ball = __ballot_sync(0xffffffffu, incl >= krem);
      const int first = ball ? __ffs(ball) - 1 : 31;
      if (lane == first) {
        unsigned above = incl - tot;
        int d = 255 - 8 * lane;
        for (int e = 0; e < 7 && d > 0; ++e, --d) {
          if (above + c[e] >= krem) break;
          above += c[e];
        }
        sh.krem -= (int)above;
        sh.prefix = pf | ((uint64_t)d << shift);
        sh.mask = mk | (0xFFull << shift);
        if ((int)sh.hist[d] == sh.krem) sh.done = 1;
      }
    }
    __syncthreads();
  }
  if (kk > 0) {
    const uint64_t pf = sh.prefix, mk = sh.mask;
    for (int i = tid; i < nc; i += nt) {
      const uint64_t k = cand[i];
      if (k != 0 && (k & mk) >= pf) {
        const int pos = atomicAdd(&sh.counter, 1);
        if (pos < K) sh.top[pos] = k;
      }
    }
  }
  __syncthreads();
  // sort the selected keys (descending) by rank; then append -inf fillers
  if (tid < kk) {
    const uint64_t k = sh.top[tid];
    int rank = 0;
    for (int i = 0; i < kk; ++i) rank += sh.top[i] > k;
    sh.sorted[rank] = k;
  }
  __syncthreads();
  if (kk < K) {
    // -inf entries in ascending flat index: row 0's non-allowed columns.  They
    // are among the first K + width columns: mark row 0's allowed ones there,
    // then warp 0 compacts the unmarked ones with ballots.
    const int range = K + width;
    for (int i = tid; i < range; i += nt) sh.fmark[i] = 0;
    __syncthreads();
    for (int j = tid; j < width; j += nt) {
      const int c = st->cols[step][0][j];
      if (c >= 0 && c < range) sh.fmark[c] = 1;
    }
    __syncthreads();
    if (tid < 32) {
      int pos = kk;
      for (int base = 0; base < range && pos < K; base += 32) {
        const int c = base + tid;
        const bool free = c < range && !sh.fmark[c];
        const unsigned m = __ballot_sync(0xffffffffu, free);
        const int r = pos + __popc(m & ((1u << tid) - 1u));
        if (free && r < K) sh.sorted[r] = cand_key(-INFINITY, (uint32_t)c);
        pos += __popc(m);
      }
    }
  }
  __syncthreads();

  // 4. decode candidates; EOS hits (max_length is never reached in 5 steps)
  if (tid < K) {
    const uint64_t k = sh.sorted[tid];
    const uint32_t flat = ~(uint32_t)(k & 0xffffffffu);
    const float score = key_float((uint32_t)(k >> 32));
    int b = (int)(flat / (uint32_t)vocab);
    if (b >= beams) { atomicOr(status, RTR_DEV_BAD_PARENT); b = 0; }
    const int tok = (int)(flat % (uint32_t)vocab);
    const int hit = tok == tb.eos;
    sh.c_score[tid] = score;
    sh.c_beam[tid] = b;
    sh.c_tok[tid] = tok;
    sh.c_hit[tid] = hit;
    // _get_running_beams_for_next_iteration: topk_log_probs + hits * -1e9
    sh.c_run[tid] = score + (hit ? -1.0e9f : -0.0f);
    // _update_finished_beams (length_penalty 0, early_stopping False)
    const int unsat = st->unsatisfied;
    const int did_finish = hit && tid < beams;
    float f = score / 1.0f + -0.0f;
    f = f + (unsat ? -0.0f : -1.0e9f);
    f = f + (did_finish ? -0.0f : -1.0e9f);
    sh.c_fin[beams + tid] = f;
  }
  if (tid < beams) sh.c_fin[tid] = sh.f_score[tid];
  __syncthreads();

  // 5. running top-beams and finished top-beams (stable: ties keep position order;
  //    scores are NaN-free, so the ranks form a permutation and fill every slot)
  if (tid < beams) { sh.n_run[tid] = 0; sh.n_fin[tid] = 0; }
  __syncthreads();
  if (tid < K) {
    const float r = sh.c_run[tid];
    int rank = 0;
    for (int i = 0; i < K; ++i) rank += (sh.c_run[i] > r) || (sh.c_run[i] == r && i < tid);
    if (rank < beams) sh.n_run[rank] = tid;
  }
  if (tid < beams + K) {
    const float f = sh.c_fin[tid];
    int rank = 0;
    for (int i = 0; i < beams + K; ++i) rank += (sh.c_fin[i] > f) || (sh.c_fin[i] == f && i < tid);
    if (rank < beams) sh.n_fin[rank] = tid;
  }
  __syncthreads();

  // 6. write the new running and finished sets
  if (tid < beams) {
    const int n = tid;
    const int j = sh.n_run[n];
    const int p = sh.c_beam[j];
    for (int t = 0; t < NSTEPS; ++t) {
      st->run_tok[n][t] = t < step ? sh.o_tok[p][t] : (t == step ? sh.c_tok[j] : tb.eos);
      st->run_par[n][t] = t < step ? sh.o_par[p][t] : (t == step ? p : -1);
    }
    st->run_score[n] = sh.c_run[j];
    st->next_tok[n] = sh.c_tok[j];
    for (int s = 0; s < 4; ++s)
      st->anc[n][s] = (s < step - 1) ? sh.o_anc[p][s] : (s == step - 1 ? p : -1);

    const int m = sh.n_fin[n];
    if (m < beams) {
      for (int t = 0; t < NSTEPS; ++t) { st->fin_tok[n][t] = sh.f_tok[m][t]; st->fin_par[n][t] = sh.f_par[m][t]; }
      st->fin_done[n] = sh.f_done[m];
      sh.nf_done[n] = sh.f_done[m];
    } else {
      const int c = m - beams, pc = sh.c_beam[c];
      for (int t = 0; t < NSTEPS; ++t) {
        st->fin_tok[n][t] = t < step ? sh.o_tok[pc][t] : (t == step ? sh.c_tok[c] : tb.eos);
        st->fin_par[n][t] = t < step ? sh.o_par[pc][t] : (t == step ? pc : -1);
      }
      st->fin_done[n] = sh.c_hit[c] && c < beams;
      sh.nf_done[n] = sh.c_hit[c] && c < beams;
    }
    st->fin_score[n] = sh.c_fin[m];
    sh.nf_score[n] = sh.c_fin[m];
  }
  __syncthreads();

  // 7. early-stop heuristic and the loop condition (utils.py:2876-2943)
  if (tid == 0) {
    float worst = INFINITY;
    for (int b = 0; b < beams; ++b) worst = fminf(worst, sh.nf_score[b]);
    const float best_running = sh.c_run[sh.n_run[0]] / 1.0f;
    bool improvable = false;
    for (int b = 0; b < beams; ++b) improvable |= best_running > (sh.nf_done[b] ? worst : -1.0e9f);
    const int unsat = st->unsatisfied && improvable;
    st->unsatisfied = unsat;
    bool all_hits = true;
    for (int i = 0; i < K; ++i) all_hits &= sh.c_hit[i] != 0;
    const bool running = unsat && !all_hits;
    if (!running && st->finished_after < 0) st->finished_after = step;
    if (step < NSTEPS - 1 && !running) atomicOr(status, RTR_DEV_STOPPED_EARLY);
    if (step == NSTEPS - 1 && running) atomicOr(status, RTR_DEV_NOT_STOPPED);
  }
}

cudaError_t beam_init() {
  return cudaFuncSetAttribute(beam_select_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                              (int)(MAX_CAND * sizeof(uint64_t)));
}

cudaError_t beam_step(BeamState* st, const float* logits, int rows, int vocab, int beams, int step,
                      const DevTables& tb, uint32_t* status, cudaStream_t stream, int users, const float2* lse) {
  dim3 grid(rows * users, TAIL_SPLITS);
  cudaError_t e = cudaSuccess;
  if (lse) {
    e = launch_pdl(PDL_TAIL, tail_lse_sum2_kernel, grid, dim3(TAIL_THREADS), 0, stream, logits, vocab, st, rows, lse);
  } else {
    e = launch_pdl(PDL_TAIL, tail_max_kernel, grid, dim3(TAIL_THREADS), 0, stream, logits, vocab, st, rows);
    if (e == cudaSuccess)
      e = launch_pdl(PDL_TAIL, tail_sum1_kernel, grid, dim3(TAIL_THREADS), 0, stream, logits, vocab, st, rows);
    if (e == cudaSuccess)
      e = launch_pdl(PDL_TAIL, tail_sum2_kernel, grid, dim3(TAIL_THREADS), 0, stream, logits, vocab, st, rows);
  }
  const int width = lookup_width_of(tb, step);
  const size_t need = (size_t)beams * width * sizeof(uint64_t);
  if (e == cudaSuccess)
    e = launch_pdl(PDL_TAIL, beam_select_kernel, dim3(users), dim3(SEL_THREADS), need, stream, st, logits, rows, vocab,
                   beams, step, tb, status);
  return e;
}

// ------------------------------------------------------------ reset / output
__global__ void beam_reset_kernel(BeamState* st, const int32_t* ids, const int32_t* L_dev, int beams) {
  const int b = threadIdx.x;
  if (b < beams) {
    for (int t = 0; t < NSTEPS; ++t) {
      st->run_tok[b][t] = -1; st->run_par[b][t] = -1;
      st->fin_tok[b][t] = -1; st->fin_par[b][t] = -1;
    }
    st->run_score[b] = b == 0 ? 0.0f : -1.0e9f;
    st->fin_score[b] = -1.0e9f;
    st->fin_done[b] = 0;
    for (int s = 0; s < 4; ++s) st->anc[b][s] = -1;
  }
  if (b == 0) {
    const int L = *L_dev;
    for (int j = 0; j < 3; ++j) st->prompt_tail[j] = ids[L - 3 + j];
    st->unsatisfied = 1;
    st->finished_after = -1;
  }
}

cudaError_t beam_reset(BeamState* st, const int32_t* ids_dev, const int32_t* L_dev, int beams,
                       cudaStream_t stream) {
  beam_reset_kernel<<<1, MAX_BEAMS, 0, stream>>>(st, ids_dev, L_dev, beams);
  return cudaGetLastError();
}

// transition_logp = scores[t][beam_indices[i][t], token[i][t]] (compute_transition_scores)
__global__ void beam_finalize_kernel(const BeamState* st, int beams, DevResult* res, const uint32_t* status) {
  st += blockIdx.x;  // one block per user
  res += blockIdx.x;
  const int i = threadIdx.x;
  if (i < beams) {
    for (int t = 0; t < NSTEPS; ++t) {
      const int tok = st->fin_tok[i][t], row = st->fin_par[i][t];
      res->token_ids[i * NSTEPS + t] = tok;
      res->beam_indices[i * NSTEPS + t] = row;
      float v = -INFINITY;
      if (row >= 0 && row < beams) {
        const int w = st->width[t];
        for (int j = 0; j < w; ++j)
          if (st->cols[t][row][j] == tok) { v = st->vals[t][row][j]; break; }
      }
      res->transition_logp[i * NSTEPS + t] = v;
    }
    res->sequence_logp[i] = st->fin_score[i];
  }
  if (i == 0) {
    res->status = *status;
    res->steps = st->finished_after + 1;
  }
}

cudaError_t beam_finalize(const BeamState* st, int beams, DevResult* res, const uint32_t* status,
                          cudaStream_t stream, int users) {
  beam_finalize_kernel<<<users, MAX_BEAMS, 0, stream>>>(st, beams, res, status);
  return cudaGetLastError();
}

__global__ void dense_fill_kernel(float* out, long n) {
  for (long i = blockIdx.x * (long)blockDim.x + threadIdx.x; i < n; i += (long)gridDim.x * blockDim.x)
    out[i] = -INFINITY;
}

__global__ void dense_scatter_kernel(const BeamState* st, int step, int beams, int vocab, float* out) {
  const int b = blockIdx.x, w = st->width[step];
  for (int j = threadIdx.x; j < w; j += blockDim.x) {
    const int col = st->cols[step][b][j];
    if (col >= 0 && col < vocab) out[(long)b * vocab + col] = st->vals[step][b][j];
  }
}

cudaError_t beam_dense_scores(const BeamState* st, int step, int beams, int vocab, float* out,
                              cudaStream_t stream) {
  dense_fill_kernel<<<148 * 4, 256, 0, stream>>>(out, (long)beams * vocab);
  dense_scatter_kernel<<<beams, 256, 0, stream>>>(st, step, beams, vocab, out);
  return cudaGetLastError();
}

// -------------------------------------------- plugin-level entry points
__global__ void lookup_kernel(DevTables tb, int step, const int64_t* ids, int rows, int cols,
                              int32_t* out, int width) {
  const int r = blockIdx.x;
  __shared__ LookupRow lr;
  if (threadIdx.x == 0) {
    long tok[3];
    const int n = (step == 0 || step == 3) ? 3 : (step < 3 ? step : 0);
    for (int j = 0; j < n; ++j) tok[j] = ids[(long)r * cols + cols - n + j];
    lr = lookup_row(tb, step, tok);
  }
  __syncthreads();
  for (int j = threadIdx.x; j < width; j += blockDim.x) out[(long)r * width + j] = lookup_col(tb, lr, j);
}

cudaError_t constraint_lookup(const DevTables& tb, int step, const int64_t* ids, int rows, int cols,
                              int32_t* out, cudaStream_t stream) {
  lookup_kernel<<<rows, 128, 0, stream>>>(tb, step, ids, rows, cols, out, lookup_width_of(tb, step));
  return cudaGetLastError();
}

// out = log_softmax(scores) + mask, split over PROC_SPLITS CTAs per row.
// Pass 1: per-slice max -> scratch[row][slice][0]; pass 2: exact row max, per-
// slice sum exp(x - max) -> scratch[row][slice][1]; pass 3: log of the summed
// slices (fixed order), -inf everywhere in the slice, then the processed
// value (x - max) - log(sum) at the allowed columns that fall in the slice.
__device__ __forceinline__ void slice_bounds(int vocab, int sp, long* lo, long* hi) {
  *lo = (long)vocab * sp / PROC_SPLITS;
  *hi = (long)vocab * (sp + 1) / PROC_SPLITS;
}

__global__ void proc_max_kernel(const float* __restrict__ scores, int vocab, float* scratch) {
  __shared__ float red[33];
  const int r = blockIdx.x, sp = blockIdx.y;
  long lo, hi;
  slice_bounds(vocab, sp, &lo, &hi);
  const float* x = scores + (long)r * vocab;
  float m = -INFINITY;
  for (long i = lo + threadIdx.x; i < hi; i += blockDim.x) m = fmaxf(m, x[i]);
  m = block_max(m, red);
  if (threadIdx.x == 0) scratch[((long)r * PROC_SPLITS + sp) * 2] = m;
}

__device__ __forceinline__ float proc_row_max(const float* scratch, int r) {
  float m = -INFINITY;
  for (int k = 0; k < PROC_SPLITS; ++k) m = fmaxf(m, scratch[((long)r * PROC_SPLITS + k) * 2]);
  return m;
}

__global__ void proc_sum_kernel(const float* __restrict__ scores, int vocab, float* scratch) {
  __shared__ float red[33];
  const int r = blockIdx.x, sp = blockIdx.y;
  long lo, hi;
  slice_bounds(vocab, sp, &lo, &hi);
  const float* x = scores + (long)r * vocab;
  const float m = proc_row_max(scratch, r);
  float s = 0.f;
  for (long i = lo + threadIdx.x; i < hi; i += blockDim.x) s += expf(x[i] - m);
  s = block_sum(s, red);
  if (threadIdx.x == 0) scratch[((long)r * PROC_SPLITS + sp) * 2 + 1] = s;
}

__global__ void proc_write_kernel(DevTables tb, int step, const int64_t* __restrict__ ids, int cols,
                                  const float* __restrict__ scores, float* __restrict__ out, int vocab,
                                  const float* scratch) {
  __shared__ LookupRow lr;
  const int r = blockIdx.x, sp = blockIdx.y;
  long lo, hi;
  slice_bounds(vocab, sp, &lo, &hi);
  const float* x = scores + (long)r * vocab;
  float* y = out + (long)r * vocab;
  const float m = proc_row_max(scratch, r);
  float s = 0.f;
  for (int k = 0; k < PROC_SPLITS; ++k) s += scratch[((long)r * PROC_SPLITS + k) * 2 + 1];
  const float L = logf(s);
  for (long i = lo + threadIdx.x; i < hi; i += blockDim.x) y[i] = -INFINITY;
  if (threadIdx.x == 0) {
    long tok[3];
    const int n = (step == 0 || step == 3) ? 3 : (step < 3 ? step : 0);
    for (int j = 0; j < n; ++j) tok[j] = ids[(long)r * cols + cols - n + j];
    lr = lookup_row(tb, step, tok);
  }
  __syncthreads();
  const int width = lookup_width_of(tb, step);
  for (int j = threadIdx.x; j < width; j += blockDim.x) {
    const int col = lookup_col(tb, lr, j);
    if (col >= lo && col < hi) y[col] = ((x[col] - m) - L) + 0.0f;
  }
}

cudaError_t constraint_process(const DevTables& tb, int step, const int64_t* ids, int rows, int cols,
                               const float* scores, float* out, int vocab, float* scratch,
                               cudaStream_t stream) {
  const dim3 grid(rows, PROC_SPLITS);
  proc_max_kernel<<<grid, TAIL_THREADS, 0, stream>>>(scores, vocab, scratch);
  proc_sum_kernel<<<grid, TAIL_THREADS, 0, stream>>>(scores, vocab, scratch);
  proc_write_kernel<<<grid, TAIL_THREADS, 0, stream>>>(tb, step, ids, cols, scores, out, vocab, scratch);
  return cudaGetLastError();
}

// ------------------------------------------- allocation-free processor
// Scratch for rtr_constraint_process_static: the per-(row, slice) max/sum
// partials live in this file-scope device array (32 KiB on every GPU that
// loads the library, for the life of the process) instead of memory the
// session allocated.  Host code must not pass `g_static_proc_scratch`
// itself to a kernel - on the host that name is only a stand-in - so its
// device address is looked up once per device with cudaGetSymbolAddress, on
// the first call with that device current, and kept (a cudaDeviceReset of the
// device afterwards would leave the kept address stale).
static __device__ __align__(256) float g_static_proc_scratch[STATIC_PROC_MAX_ROWS * PROC_SPLITS * 2];

static std::mutex g_static_proc_mutex;
static float* g_static_proc_ptr[STATIC_PROC_MAX_DEVICES] = {};

cudaError_t constraint_process_static(const DevTables& tb, int step, const int64_t* ids, int rows, int cols,
                                      const float* scores, float* out, int vocab, cudaStream_t stream) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev < 0 || dev >= STATIC_PROC_MAX_DEVICES || rows < 1 || rows > STATIC_PROC_MAX_ROWS)
    return cudaErrorInvalidValue;
  float* scratch = nullptr;
  {
    std::lock_guard<std::mutex> lock(g_static_proc_mutex);
    if (!g_static_proc_ptr[dev]) {
      // first call on this device (the current one): resolve the array's address
      void* p = nullptr;
      e = cudaGetSymbolAddress(&p, g_static_proc_scratch);
      if (e != cudaSuccess) return e;
      g_static_proc_ptr[dev] = static_cast<float*>(p);
    }
    scratch = g_static_proc_ptr[dev];
  }
  // every slot a launch reads is written earlier in the same launch sequence,
  // so nothing left by a previous call needs clearing
  return constraint_process(tb, step, ids, rows, cols, scores, out, vocab, scratch, stream);
}

}  // namespace rtr
