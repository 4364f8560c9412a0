// gr_beam_step.cu — fused constrained beam-search step for B200 (sm_100a).
//
// A step is three kernels on the caller's stream:
//   row_meta_kernel   one thread per row (one row = one beam of one request):
//                     the row's 128-byte record (node, cum, CSR range, child
//                     tokens of small nodes, temperature) and the per-step
//                     resets (request bound, list lengths);
//   step kernel       persistent CTAs walk the rows: every logit row is streamed
//                     once through a ring of shared-memory stages filled by
//                     cp.async.bulk (one elected thread, mbarrier completion)
//                     while the consumer warps keep an online max / sum-exp
//                     (vLLM's full-vocab log_softmax normaliser,
//                     sampler.py:300-301); the row's candidates (trie children
//                     from a shared-memory copy of the row's child window, or
//                     a bounded top-k of the streamed values) are scored
//                     score = cum + (y - lse) (serving_engine.py:511, 533),
//                     filtered against the request's running 2B-th best key,
//                     cut to 2B and appended to the request's candidate list.
//                     Two kernels: fused_step_ws_kernel (gr_step_ws.cuh, warp-
//                     specialised producer / streaming / row-end warps) and
//                     fused_step_kernel below (all consumer warps do every
//                     phase; penalties and reference-literal top-K);
//   merge_kernel      one CTA per request: the canonical top-2B of its list,
//                     the new beams, child nodes and the forked token table
//                     (serving_engine.py:566-590).
// Kernels wait for one another only through stream order (programmatic
// dependent launch overlaps prologues); every mbarrier wait is bounded.

#include <cstdint>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <cuda_runtime.h>
#include <mutex>
#include <type_traits>
#include <utility>

#include "../../include/gr_beam.h"
#include "gr_nvtx.h"
#include "gr_device.cuh"

namespace gr {

constexpr int kModeProcessed = 1;

// Optional per-phase cycle counters (compile with -DGR_PHASE_PROFILE; off in
// the product build).  Thread 0 of every CTA adds clock64 deltas per phase
// into shared memory and flushes them to g_phase when the CTA ends.
#ifdef GR_PHASE_PROFILE
constexpr int kProfSlots = 16;
__device__ unsigned long long g_phase[1024][kProfSlots];
#define GR_PROF_T(var) const long long var = clock64()
#define GR_PROF_ADD(slot, t0) \
  do { if (threadIdx.x == 0) S.v->prof[slot] += clock64() - (t0); } while (0)
#define GR_PROF_CNT(slot) \
  do { if (threadIdx.x == 0) S.v->prof[slot] += 1; } while (0)
#define GR_PROF_VAL(slot, val) \
  do { if (threadIdx.x == 0) S.v->prof[slot] += (val); } while (0)
#define GR_PROF_INIT() \
  do { if (threadIdx.x < kProfSlots) S.v->prof[threadIdx.x] = 0; } while (0)
#define GR_PROF_FLUSH() \
  do { if (threadIdx.x == 0) for (int q = 0; q < kProfSlots; ++q) g_phase[blockIdx.x][q] += S.v->prof[q]; } while (0)
#else
#define GR_PROF_T(var)
#define GR_PROF_ADD(slot, t0) do { } while (0)
#define GR_PROF_CNT(slot) do { } while (0)
#define GR_PROF_VAL(slot, val) do { } while (0)
#define GR_PROF_INIT() do { } while (0)
#define GR_PROF_FLUSH() do { } while (0)
#endif

struct Params {
  // descriptor
  int R, NB, B, V, VL, voff;
  int vstride;   // local column j holds token voff + j * vstride
  long long row_stride;
  int mode, K, eos, T, N;
  // inputs
  const void* logits;
  const float* cum;
  const int* node;
  const long long* row_ptr;
  const int* child_tok;
  const int* child_node;
  const float* temp;
  const float* rep;
  const float* pres;
  const float* freq;
  const int* hist;
  // outputs
  float* cand_score;
  int* cand_token;
  int* cand_parent;
  float* sel_score;
  int* sel_token;
  int* sel_parent;
  int* sel_node;
  float* eos_score;
  int* hist_out;
  float* lse_out;
  int* err;
  // workspace
  unsigned long long* tau;     // [R] running lower bound of the request's 2B-th key
  unsigned int* row_counter;   // next row to hand out (rows taken dynamically by the CTAs)
  unsigned int* req_hist;      // [R][kReqHistBins] emitted keys per score bin (large 2B only, else null)
  unsigned int* rowcnt;        // [R*NB] keys in each row's slot
  int* meta;                   // [R*NB][kMetaWords] row metadata resolved by row_meta_kernel
  unsigned long long* buf;     // [R*NB][2B] per-row candidate slots
  int* pen_tab;                // [R*NB][2][tabw] each row's penalised local columns, then their processed
                               // values (bits), valid entries first, -1 after (selecting kernel, or null)
  int tabw;                    // entries per array: the history length rounded up to 32
  // derived
  int k2;        // 2B candidates
  int kk;        // streamed keep count: max(2B, K) + slack
  int sub_vecs;  // streamed rows: 16-byte vectors between key-list capacity checks
  int pen;       // penalty pointers present
  int stages;
  int bm_words;
  int tab_cap;   // penalty table entries (>= the history length)
  int win_bytes; // child window bytes (0: no constrained rows in the step)
  int partial_only;   // 1: write (max, sumexp) partials only (vocab-sharded phase 1)
  int stall_copies;   // test hook: the producer issues no copies, so the bounded waits run out
  int clear_err;      // GR_STEP_CLEAR_ERR: row_meta_kernel zeroes *err; bad nodes are reported by the merge
  float2* partials;
  const float* lse_in;            // vocab-sharded phase 2: the rows' global normaliser (no streaming)
  unsigned long long* keys_out;   // merge writes the sorted top-2B keys [R][2B] (zero padded) instead
  // merge input grid: request r's slot s sits at buf + (r * slot_sr + s * slot_sb) * 2B and
  // holds up to slot_cap keys.  The step's own lists are one slot per request
  // (slot_rows 1, the rows' keys appended at rowcnt[r * NB]).
  int slot_rows;
  long long slot_sr, slot_sb;
  int slot_cap;
};

// Vocabulary of the local columns: column j holds token voff + j * vstride
// (vstride 1: a contiguous slice; vstride = shards: a strided split).
// Local column of token t, or -1 when this shard does not hold it.
__device__ __forceinline__ int col_of(const Params& P, int t) {
  const int d = t - P.voff;
  if (d < 0) return -1;
  if (P.vstride == 1) return d < P.VL ? d : -1;
  const int j = d / P.vstride;
  return (j * P.vstride == d && j < P.VL) ? j : -1;
}
__device__ __forceinline__ int tok_of(const Params& P, int j) { return P.voff + j * P.vstride; }
// The first local column whose token is >= t, and the last one whose token is
// <= t (-1 when there is none).
__device__ __forceinline__ int col_ceil(const Params& P, int t) {
  const int d = t - P.voff;
  return (d <= 0) ? 0 : (d + P.vstride - 1) / P.vstride;
}
__device__ __forceinline__ int col_floor(const Params& P, int t) {
  const int d = t - P.voff;
  return (d < 0) ? -1 : d / P.vstride;
}

// Shared-memory layout (dynamic shared memory).  Every piece but the ring sits
// at a compile-time offset, so accesses need no pointer arithmetic at run time;
// the optional penalty pieces follow, and the ring of bulk-copy stages is last.
// Row metadata record (kMetaWords 32-bit words), resolved for every row by
// row_meta_kernel before the fused kernel so that a row's setup is one
// prefetched load instead of a chain of dependent loads.
// Request score histogram: bins of 1/16 nat below the request's first beam's
// cum, kept for steps with 2B >= kReqHistMinK2.  Rows add the keys they emit;
// the first bin where the count from the top reaches 2B bounds the request's
// 2B-th key from below (the union of all rows' lists, not one row's).
constexpr int kReqHistBins = 1024;
constexpr int kReqHistMinK2 = 512;
constexpr float kReqHistScale = 16.0f;

constexpr int kMetaSmall = 16;                  // child tokens kept for small nodes
constexpr int kMetaWords = 32;                  // 128 bytes
enum MetaWord {
  kMNode = 0, kMCum = 1, kMC0 = 2, kMC1 = 3, kMLo = 4, kMHi = 5,   // node, cum, CSR range, child token bounds
  kMTeff = 6, kMRteff = 7,                                          // effective temperature and its reciprocal
  kMRow = 8, kMR = 9, kMB = 10,                                     // row, request, beam
  kMRef = 11,                                                       // the request's first beam's cum
  kMToks = 12,                                                      // child tokens of small nodes (16 words)
  kMTauLo = 28, kMTauHi = 29,                                       // request threshold (filled on chip)
  kMBad = 30                                                        // the row's node id was out of range
};
static_assert(kMToks + kMetaSmall <= kMTauLo, "record layout");

struct Scalars {
  int meta[kMetaWords];        // the current row's record
  uint32_t cnt;
  uint32_t ntab;
  int overflow;
  int abort;
  int abort_snap;              // the consumers' abort decision at the row end (one value for all)
  int last;
  int discard;
  uint32_t base;
  float lse;
  float m_tot;
  float s_tot;
  float thr_y;
  uint64_t thr_key;
  uint64_t min_key;
  uint64_t tau_pref;
  float lse_w[kWarps];         // streamed rows: each warp's log-sum-exp so far (cta_lse_bound)
  long long issued;
  int producer_done;
#ifdef GR_PHASE_PROFILE
  unsigned long long prof[kProfSlots];
#endif
};

__host__ __device__ constexpr size_t align128(size_t x) { return (x + 127) & ~size_t(127); }

constexpr size_t kOffKeys = 0;
constexpr size_t kOffSel = kOffKeys + align128(size_t(kKeyCap) * 8);
constexpr size_t kOffRed = kOffSel + align128(sizeof(SelectScratch));
constexpr size_t kOffBars = kOffRed + align128(kWarps * 8);
constexpr size_t kOffScal = kOffBars + align128(kMaxStages * 16);
// the per-step pieces follow: the child window (steps with a catalog), the
// penalty bitmap and table (steps with penalties), the ring
constexpr size_t kOffWin = kOffScal + align128(sizeof(Scalars));

__host__ __device__ inline size_t pen_bytes(int bm_words, int tab_cap, int pen) {
  return pen ? align128(size_t(bm_words) * 4) + align128(size_t(tab_cap) * 12) : 0;
}

__host__ __device__ inline size_t smem_bytes(int stages, int win_bytes, int bm_words, int tab_cap, int pen) {
  return kOffWin + align128(size_t(win_bytes)) + pen_bytes(bm_words, tab_cap, pen) +
         align128(size_t(stages) * kStageBytes);
}

extern __shared__ __align__(128) unsigned char g_smem[];

struct Smem {
  unsigned char* ring;
  uint64_t* keys;
  unsigned char* win;   // raw logits of the child window
  uint32_t* bitmap;
  int* tab_tok;
  float* tab_xp;
  float* tab_y;
  SelectScratch* sel;
  float* red_m;
  float* red_s;
  uint64_t* full;
  uint64_t* empty;
  Scalars* v;
};

// By-value view of the layout; build it inside each function that needs it.
__device__ __forceinline__ Smem smem_view(const Params& P) {
  Smem S;
  S.keys = reinterpret_cast<uint64_t*>(g_smem + kOffKeys);
  S.win = g_smem + kOffWin;
  S.sel = reinterpret_cast<SelectScratch*>(g_smem + kOffSel);
  S.red_m = reinterpret_cast<float*>(g_smem + kOffRed);
  S.red_s = reinterpret_cast<float*>(g_smem + kOffRed + kWarps * 4);
  S.full = reinterpret_cast<uint64_t*>(g_smem + kOffBars);
  S.empty = S.full + kMaxStages;
  S.v = reinterpret_cast<Scalars*>(g_smem + kOffScal);
  const size_t var = kOffWin + align128(size_t(P.win_bytes));
  S.bitmap = reinterpret_cast<uint32_t*>(g_smem + var);
  const size_t tab = var + align128(size_t(P.bm_words) * 4);
  S.tab_tok = reinterpret_cast<int*>(g_smem + tab);
  S.tab_xp = reinterpret_cast<float*>(g_smem + tab + size_t(P.tab_cap) * 4);
  S.tab_y = reinterpret_cast<float*>(g_smem + tab + size_t(P.tab_cap) * 8);
  S.ring = g_smem + var + pen_bytes(P.bm_words, P.tab_cap, P.pen);
  return S;
}

// Row geometry: [0, head) and [tail_start, VL) are read with plain loads; the
// 16-byte aligned body in between goes through the bulk-copy ring.
struct Geom {
  const char* rowp;
  const char* body;
  long long body_bytes;
  int head;
  int tail_start;
  int nchunks;
};

template <int ES, int SB = kStageBytes>
__device__ __forceinline__ Geom row_geom(const Params& P, int row) {
  Geom g;
  g.rowp = static_cast<const char*>(P.logits) + static_cast<size_t>(row) * static_cast<size_t>(P.row_stride) * ES;
  const uintptr_t a = reinterpret_cast<uintptr_t>(g.rowp);
  const uintptr_t e = a + static_cast<uintptr_t>(P.VL) * ES;
  const uintptr_t a0 = (a + 15) & ~uintptr_t(15);
  const uintptr_t a1 = e & ~uintptr_t(15);
  if (a1 <= a0) {
    g.body = g.rowp;
    g.body_bytes = 0;
    g.head = P.VL;
    g.tail_start = P.VL;
    g.nchunks = 0;
  } else {
    g.body = reinterpret_cast<const char*>(a0);
    g.body_bytes = static_cast<long long>(a1 - a0);
    g.head = static_cast<int>((a0 - a) / ES);
    g.tail_start = static_cast<int>((a1 - a) / ES);
    g.nchunks = static_cast<int>((g.body_bytes + SB - 1) / SB);
  }
  return g;
}

// b-major order: the first rows taken are the requests' best beams, which
// raise the per-request thresholds early.
__device__ __forceinline__ int row_of_seq(const Params& P, int seq) {
  const int b = seq / P.R;
  const int r = seq - b * P.R;
  return r * P.NB + b;
}

__device__ __forceinline__ int row_of_iter(const Params& P, int it) {
  return row_of_seq(P, blockIdx.x + it * gridDim.x);
}

__device__ __forceinline__ float eff_temperature(const Params& P, int r) {
  if (P.temp == nullptr) return 1.0f;
  const float t = P.temp[r];
  return (t < 1e-5f) ? 1.0f : t;
}

// vLLM penalties for one token seen `cnt` times in the output history
// (model_executor/layers/utils.py:51-89): repetition, then frequency, then
// presence, each rounded to float32 (no fused multiply-add).
__device__ __forceinline__ float penalise(float x, int cnt, float rep, float pres, float freq) {
  x = (x > 0.0f) ? __fdiv_rn(x, rep) : __fmul_rn(x, rep);
  x = __fsub_rn(x, __fmul_rn(freq, static_cast<float>(cnt)));
  x = __fsub_rn(x, pres);
  return x;
}

// Lowest y a streamed element needs to reach the request bound tau: its score
// cum + (y - lse) must reach tau's score, and lse >= L.  -inf without a bound.
__device__ __forceinline__ float tau_floor_value(uint64_t tau, float cum, float L) {
  if (tau == 0ull || !(L > -kInf && L < kInf)) return -kInf;
  const float ts = key_score(tau);
  const float f = ts - cum + L;
  if (!(f > -kInf && f < kInf)) return -kInf;
  // margin for y vs the exact quotient, the approximate logarithms and the
  // roundings of the score sum (relative to the magnitudes of its terms)
  return f - 1.0e-5f * (fabsf(f) + fabsf(ts) + fabsf(cum) + fabsf(L)) - 1e-30f;
}

struct RowCtx {
  int row, r, b, node;
  int c0, c1;          // CSR edge range of the node (c0 == c1: none)
  int lo_tok;          // first child token
  bool dense;          // children are exactly the tokens lo_tok .. lo_tok + (c1 - c0) - 1
  int wlo, whi;        // window [wlo, whi] in local columns (empty if wlo > whi)
  bool stream;         // unconstrained or reference-literal
  bool constrained;
  bool pen_active;     // penalty table in use for this row
  bool excl;           // processed mode: penalised tokens come from the table
  float teff, rteff;
  float rep, pres, freq;
  float cum;
};

// kExtTable: the kernel keeps the row's penalty table outside the common
// shared-memory pieces (and no column bitmap); lookups scan that table.
template <typename TL, bool kExtTable = false>
struct Step {
  using Tr = LogitTraits<TL>;
  static constexpr int ES = sizeof(TL);
  static constexpr int EPV = Tr::kPerVec;

  const Params& P;
  int win_off = 0;            // byte offset of the current row's window from the first window
  const int* rec = nullptr;   // the current row's metadata record (shared memory)
  // kExtTable: the row's penalty table (penalised local columns, their
  // processed values and count), set per row by the kernel
  const int* ext_tok = nullptr;
  const float* ext_y = nullptr;
  const int* ext_n = nullptr;
  __device__ __forceinline__ explicit Step(const Params& p) : P(p) {}

  __device__ __forceinline__ float load_logit(const RowCtx& c, int tl) const {
    const TL* rowp = reinterpret_cast<const TL*>(static_cast<const char*>(P.logits) +
                                                 static_cast<size_t>(c.row) * static_cast<size_t>(P.row_stride) * ES);
    return Tr::load1(rowp + tl);
  }

  static constexpr int kWinTok = kWinBytes / ES;

  __device__ __forceinline__ unsigned char* win() const { return g_smem + kOffWin + win_off; }
  __device__ __forceinline__ void win_store(int i, float x) const {
    if constexpr (ES == 4) {
      reinterpret_cast<float*>(win())[i] = x;
    } else if constexpr (std::is_same_v<TL, __nv_bfloat16>) {
      reinterpret_cast<unsigned short*>(win())[i] = static_cast<unsigned short>(__float_as_uint(x) >> 16);
    } else {
      reinterpret_cast<__half*>(win())[i] = __float2half_rn(x);
    }
  }
  __device__ __forceinline__ float win_load(int i) const {
    if constexpr (ES == 4) {
      return reinterpret_cast<const float*>(win())[i];
    } else if constexpr (std::is_same_v<TL, __nv_bfloat16>) {
      return __uint_as_float(static_cast<uint32_t>(reinterpret_cast<const unsigned short*>(win())[i]) << 16);
    } else {
      return __half2float(reinterpret_cast<const __half*>(win())[i]);
    }
  }

  __device__ __forceinline__ bool flagged(const RowCtx& c, int tl) const {
    if constexpr (kExtTable) {
      return c.pen_active;
    } else {
      const Smem S = smem_view(P);
      return c.pen_active && ((S.bitmap[tl >> 5] >> (tl & 31)) & 1u);
    }
  }

  __device__ __forceinline__ int table_find(int tl) const {
    if constexpr (kExtTable) {
      const int n = *ext_n;
      for (int j = 0; j < n; ++j)
        if (ext_tok[j] == tl) return j;
    } else {
      const Smem S = smem_view(P);
      const int n = static_cast<int>(S.v->ntab);
      for (int j = 0; j < n; ++j)
        if (S.tab_tok[j] == tl) return j;
    }
    return -1;
  }

  // Exact value in the log-prob domain for local column tl whose raw logit is x.
  __device__ __forceinline__ float exact_y(const RowCtx& c, float x, int tl) const {
    if (P.mode == kModeProcessed) {
      if (c.excl && flagged(c, tl)) {
        const int j = table_find(tl);
        if (j >= 0) {
          if constexpr (kExtTable) return ext_y[j];
          else return smem_view(P).tab_y[j];
        }
      }
      return (c.teff == 1.0f) ? x : __fdiv_rn(x, c.teff);
    }
    return x;
  }

  // ---- per-element streaming work ----------------------------------------
  // Online (max, sumexp) update with n values; -inf values contribute nothing.
  template <int N>
  __device__ __forceinline__ void lse_update(const float* y, float& m, float& s) const {
    float vmax = y[0];
#pragma unroll
    for (int i = 1; i < N; ++i) vmax = fmaxf(vmax, y[i]);
    if (vmax > m) {
      s = s * fast_exp2((m - vmax) * kLog2e);
      m = vmax;
    }
    if (m > -kInf) {
      const float mb = m * kLog2e;
#pragma unroll
      for (int i = 0; i < N; ++i) s += fast_exp2(fmaf(y[i], kLog2e, -mb));
    }
  }

  // Process N consecutive columns starting at local column tb (x = raw values,
  // valid = lane holds real data).  Warp-uniform call.
  // y_floor: streamed rows skip elements below it (-inf: none); see tau_floor().
  // lse = false: (m, s) already hold these columns; only the candidate part runs.
  template <int N>
  __device__ __forceinline__ void process(const RowCtx& c, const float* x, int tb, bool valid, float& m, float& s,
                                          float thr_y, uint64_t thr_key, float y_floor = -__builtin_huge_valf(),
                                          bool lse = true) const {
    const Smem S = smem_view(P);
    float y[N];
#pragma unroll
    for (int i = 0; i < N; ++i) y[i] = (P.mode == kModeProcessed) ? x[i] * c.rteff : x[i];
    uint32_t fl = 0;
    if (c.excl && valid) {
      const int w = tb >> 5, sh = tb & 31;
      uint64_t bits = S.bitmap[w];
      if (w + 1 < P.bm_words) bits |= static_cast<uint64_t>(S.bitmap[w + 1]) << 32;
      fl = static_cast<uint32_t>(bits >> sh) & ((N >= 32) ? 0xFFFFFFFFu : ((1u << N) - 1u));
      if (fl) {
#pragma unroll
        for (int i = 0; i < N; ++i)
          if ((fl >> i) & 1u) y[i] = -kInf;
      }
    }
    if (valid && lse) {
      lse_update<N>(y, m, s);
      if (c.constrained && tb + N > c.wlo && tb <= c.whi) {
#pragma unroll
        for (int i = 0; i < N; ++i) {
          const int tl = tb + i;
          if (tl >= c.wlo && tl <= c.whi) win_store(tl - c.wlo, x[i]);
        }
      }
    }
    if (c.stream) {
      const float thr_e = fmaxf(thr_y, y_floor);
      bool any = false;
#pragma unroll
      for (int i = 0; i < N; ++i) any |= valid && !((fl >> i) & 1u) && (y[i] >= thr_e);
      if (__any_sync(0xFFFFFFFFu, any)) {
        const uint32_t fbase = static_cast<uint32_t>(c.b) * static_cast<uint32_t>(P.V) +
                               static_cast<uint32_t>(tok_of(P, tb));
        uint64_t kv[N];
        uint32_t mask = 0;
#pragma unroll
        for (int i = 0; i < N; ++i) {
          kv[i] = 0;
          if (valid && !((fl >> i) & 1u) && (y[i] >= thr_e)) {
            const float ye = (P.mode == kModeProcessed && c.teff != 1.0f) ? __fdiv_rn(x[i], c.teff) : x[i];
            kv[i] = make_key(ye, fbase + static_cast<uint32_t>(i * P.vstride));
            if (kv[i] >= thr_key) mask |= 1u << i;
          }
        }
        warp_append_n<N>(mask, kv, S.keys, &S.v->cnt, kKeyCap, &S.v->overflow);   // one reservation per warp
      }
    }
  }

  // Log-sum-exp of the columns the CTA has seen so far, a lower bound of the
  // row's.  Each warp publishes its own in lse_w (one float, reset to -inf at
  // the row start); the other warps' values may be a few stages old and are
  // still lower bounds of their final sums.  (m, s) are the calling thread's
  // running max and sum.  Warp-collective; -inf when nothing is known yet.
  __device__ __forceinline__ float cta_lse_bound(float m, float s, float* lse_w) const {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    float M = m;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) M = fmaxf(M, __shfl_xor_sync(0xFFFFFFFFu, M, o));
    float t = (m == -kInf) ? 0.0f : s * fast_exp2((m - M) * kLog2e);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) t += __shfl_xor_sync(0xFFFFFFFFu, t, o);
    const float Lw = (M > -kInf && t > 0.0f && t < kInf) ? M + __logf(t) : -kInf;
    float Lo[kWarps];
#pragma unroll
    for (int w = 0; w < kWarps; ++w) Lo[w] = (w == warp) ? Lw : lse_w[w];
    if (lane == 0) lse_w[warp] = Lw;
    float Lm = -kInf;
#pragma unroll
    for (int w = 0; w < kWarps; ++w) Lm = fmaxf(Lm, Lo[w]);
    if (!(Lm > -kInf && Lm < kInf)) return -kInf;
    float tot = 0.0f;
#pragma unroll
    for (int w = 0; w < kWarps; ++w) tot += fast_exp2((Lo[w] - Lm) * kLog2e);
    return Lm + __logf(tot);
  }

  __device__ __forceinline__ float tau_floor(const RowCtx& c, uint64_t tau, float L) const {
    return tau_floor_value(tau, c.cum, L);
  }

  // ---- selection helpers ------------------------------------------------------
  // The key list's length as every thread reads it between two barriers: the
  // same value everywhere (the decisions taken on it are uniform), and no
  // thread appends again before all of them have read it.
  __device__ __forceinline__ int list_len_sync() const {
    const Smem S = smem_view(P);
    csync();
    const int n = static_cast<int>(S.v->cnt);
    csync();
    return n;
  }

  // Reduce the shared key list to its best k (k < cnt).  Returns the cut.
  __device__ Cut shrink_to(int k) {
    const Smem S = smem_view(P);
    GR_PROF_T(t0);
    const int n = min(static_cast<int>(S.v->cnt), kKeyCap);
    uint64_t* keys = S.keys;
    Cut cut = cta_radix_select([keys](int i) { return keys[i]; }, n, k, S.sel);
    cta_compact(S.keys, n, cut, &S.v->cnt);
    GR_PROF_ADD(8, t0);
    GR_PROF_CNT(9);
    return cut;
  }

  __device__ void raise_tau(int r, uint64_t floor_key) {
    const Smem S = smem_view(P);
    if (threadIdx.x == 0) {
      atomicMax(P.tau + r, static_cast<unsigned long long>(floor_key));
      if (floor_key > S.v->thr_key) S.v->thr_key = floor_key;
    }
    csync();
  }

  __device__ uint64_t min_key_of_list() {
    const Smem S = smem_view(P);
    const int n = min(static_cast<int>(S.v->cnt), kKeyCap);
    uint64_t mn = ~0ull;
    for (int i = threadIdx.x; i < n; i += kThreads) mn = (S.keys[i] < mn) ? S.keys[i] : mn;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const uint64_t v = __shfl_xor_sync(0xFFFFFFFFu, mn, o);
      mn = v < mn ? v : mn;
    }
    if (threadIdx.x == 0) S.v->min_key = ~0ull;
    csync();
    if (lane_id() == 0) atomicMin(reinterpret_cast<unsigned long long*>(&S.v->min_key), mn);
    csync();
    const uint64_t res = S.v->min_key;
    csync();
    return res;
  }

  // ---- row-end candidate formation -----------------------------------------
  // Load window entries [i, i+8) (i a multiple of 8) as floats.
  __device__ __forceinline__ void win_load8(int i, float* x) const {
    if constexpr (ES == 4) {
      const uint4 a = reinterpret_cast<const uint4*>(win())[i >> 2];
      const uint4 b = reinterpret_cast<const uint4*>(win())[(i >> 2) + 1];
      x[0] = __uint_as_float(a.x); x[1] = __uint_as_float(a.y); x[2] = __uint_as_float(a.z); x[3] = __uint_as_float(a.w);
      x[4] = __uint_as_float(b.x); x[5] = __uint_as_float(b.y); x[6] = __uint_as_float(b.z); x[7] = __uint_as_float(b.w);
    } else {
      Tr::unpack(reinterpret_cast<const uint4*>(win())[i >> 3], x);
    }
  }

  // Ordered integer of window entry i (larger = larger value; 16 significant
  // bits for 2-byte logits, 32 for f32) and its inverse.
  __device__ __forceinline__ uint32_t win_ord(int i) const {
    if constexpr (ES == 4) {
      return f32_to_ord(reinterpret_cast<const float*>(win())[i]);
    } else {
      const uint32_t u = reinterpret_cast<const unsigned short*>(win())[i];
      return (u & 0x8000u) ? (~u & 0xFFFFu) : (u | 0x8000u);
    }
  }
  __device__ __forceinline__ float ord_value(uint32_t o) const {
    if constexpr (ES == 4) {
      return ord_to_f32(o);
    } else {
      const uint32_t u = (o & 0x8000u) ? (o & 0x7FFFu) : (~o & 0xFFFFu);
      if constexpr (std::is_same_v<TL, __nv_bfloat16>) return __uint_as_float(u << 16);
      else return __half2float(__ushort_as_half(static_cast<unsigned short>(u)));
    }
  }
  // Key of child j at window index i: value first, then the lower child index.
  __device__ __forceinline__ uint64_t win_value_key(int i, int j) const {
    if constexpr (ES == 4) {
      return (static_cast<uint64_t>(win_ord(i)) << 32) | static_cast<uint64_t>(0xFFFFFFFFu - static_cast<uint32_t>(j));
    } else {
      return static_cast<uint64_t>((win_ord(i) << 16) | (0xFFFFu - static_cast<uint32_t>(j))) << 32;
    }
  }
  __device__ __forceinline__ float value_of_key(uint64_t k) const {
    if constexpr (ES == 4) return ord_value(static_cast<uint32_t>(k >> 32));
    else return ord_value(static_cast<uint32_t>(k >> 48));
  }

  // Score child j (CSR position within the node, token tok) of a catalog row.
  // Its key carries parent * V + j: children are sorted by token, so this
  // orders ties exactly as parent * V + token does, and the merge reads the
  // token and the child node at c0 + j without a search.
  __device__ __forceinline__ uint64_t child_key(const RowCtx& c, int tok, int j, float x, float lse,
                                                uint32_t fb) const {
    const float y = exact_y(c, x, col_of(P, tok));
    float sc = __fadd_rn(c.cum, __fsub_rn(y, lse));
    if (tok == P.eos) {
      if (P.eos_score) P.eos_score[c.row] = sc;
      sc = -kInf;
    }
    return make_key(sc, fb + static_cast<uint32_t>(j));
  }

  __device__ void constrained_candidates(const RowCtx& cref, float lse) {
    const Smem S = smem_view(P);
    const RowCtx c = cref;
    const int c0 = c.c0, c1 = c.c1, deg = c1 - c0;
    const uint32_t fb = static_cast<uint32_t>(c.b) * static_cast<uint32_t>(P.V);
    // Scores of all children are compared against the threshold in float
    // first; only the (rare) passers build keys and take part in the append.
    // An exact float test is enough: key >= thr implies score >= score(thr).
    const bool processed_div = (P.mode == kModeProcessed) && (c.excl || c.teff != 1.0f);
    // the window path: a contiguous shard holding every child of a dense node
    // in its child window, child j at window entry d0 + j
    const int first = c.lo_tok - P.voff;
    const bool dense_window = P.vstride == 1 && c.dense && !processed_div && first >= c.wlo &&
                              first + deg - 1 <= c.whi;
    const int d0 = first - c.wlo;               // window index of the first child
    static_assert(kBatch == kThreads * 8, "dense path: one 8-entry group per thread per batch");
    bool dense_done = false;
    constexpr int kG = 4;   // the one-pass dense scan covers kG * kBatch window entries
    // an EOS child scores -inf in the pool: the value bound then takes one child more
    const int eos_j = (P.eos >= 0) ? P.eos - c.lo_tok : -1;
    const int ksel = P.k2 + ((eos_j >= 0 && eos_j < deg) ? 1 : 0);
    for (int attempt = 0; attempt < 2 && !dense_done && dense_window && d0 + deg <= kG * kBatch; ++attempt) {
      if ((S.v->thr_key == 0ull || attempt == 1) && deg > ksel) {
        // a weak bound: tighten it with the row's own 2B-th best child value
        // (the (2B+1)-th when one child is EOS).  Scores are monotone in the
        // value, so every child scoring at least that value's score is kept,
        // and at least 2B children other than EOS do.
        // (only the value bits are resolved: the bound needs the value alone)
        const Cut vc = cta_radix_select([this, d0](int j) { return win_value_key(d0 + j, j); }, deg, ksel, S.sel,
                                        ES == 4 ? 32 : 48);
        if (threadIdx.x == 0) {
          const float xt = value_of_key(vc.floor_key());
          const float st = __fadd_rn(__fadd_rn(c.cum, __fsub_rn(xt, lse)), 0.0f);
          const uint64_t tk = static_cast<uint64_t>(f32_to_ord(st)) << 32;
          if (tk > S.v->thr_key) S.v->thr_key = tk;
        }
        csync();
      }
      // one pass over every child with a single reservation per warp; if the key
      // list overflows, the row is redone (tighter bound, or the batched loop)
      const uint64_t thr = S.v->thr_key;
      const float thr_s = thr ? key_score(thr) : -kInf;
      // dense children score as the window value (no temperature, no table):
      // the key arithmetic runs branch-free for all of them; EOS keeps a -inf
      // score and records its completion score
      uint32_t pm[kG];
      uint32_t cnt_t = 0;
#pragma unroll
      for (int g = 0; g < kG; ++g) {
        pm[g] = 0;
        const int w0 = g * kBatch + static_cast<int>(threadIdx.x) * 8;
        const int i0 = w0 - d0;
        if (w0 < d0 + deg) {
          float x[8];
          win_load8(w0, x);
          float xm = x[0];
#pragma unroll
          for (int i = 1; i < 8; ++i) xm = fmaxf(xm, x[i]);
          // scores are monotone in the value: a group whose best score misses the
          // bound has no candidate (only its EOS child, if any, needs a look)
          const bool eos_here = eos_j >= i0 && eos_j < i0 + 8;
          if (eos_here || !(__fadd_rn(c.cum, __fsub_rn(xm, lse)) < thr_s)) {
#pragma unroll
            for (int i = 0; i < 8; ++i) {
              const int j = i0 + i;
              const bool in = (j >= 0) && (j < deg);
              float sc = __fadd_rn(c.cum, __fsub_rn(x[i], lse));
              if (in && j == eos_j) {
                if (P.eos_score) P.eos_score[c.row] = sc;
                sc = -kInf;
              }
              if (in && make_key(sc, fb + static_cast<uint32_t>(j)) >= thr) pm[g] |= 1u << i;
            }
          }
        }
        cnt_t += static_cast<uint32_t>(__popc(pm[g]));
      }
      uint32_t pos = warp_reserve(cnt_t, &S.v->cnt);
#pragma unroll
      for (int g = 0; g < kG; ++g) {
        if (pm[g]) {
          const int w0 = g * kBatch + static_cast<int>(threadIdx.x) * 8;
          const int i0 = w0 - d0;
          float x[8];
          win_load8(w0, x);
#pragma unroll
          for (int i = 0; i < 8; ++i) {
            if ((pm[g] >> i) & 1u) {
              const int j = i0 + i;
              const float sc = (j == eos_j) ? -kInf : __fadd_rn(c.cum, __fsub_rn(x[i], lse));
              if (pos < static_cast<uint32_t>(kKeyCap))
                S.keys[pos] = make_key(sc, fb + static_cast<uint32_t>(j));
              else
                S.v->overflow = 1;
              ++pos;
            }
          }
        }
      }
      csync();
      if (S.v->overflow == 0) {
        dense_done = true;
      } else {
        csync();
        if (threadIdx.x == 0) {
          S.v->cnt = 0;
          S.v->overflow = 0;
        }
        csync();
      }
    }
    if (dense_done) {
      // every child was scored in the one pass
    } else if (dense_window) {
      // child j sits at window index d0 + j: 8 window entries per thread per 16-byte load
      for (int base = 0; base < d0 + deg; base += kBatch) {
        const uint64_t thr = S.v->thr_key;
        const float thr_s = thr ? key_score(thr) : -kInf;
        // other rows of the request raise its bound meanwhile: read it for the next batch
        uint64_t tau_g = 0;
        if (threadIdx.x == 0 && base + kBatch < d0 + deg) tau_g = *reinterpret_cast<volatile unsigned long long*>(P.tau + c.r);
        const int w0 = base + static_cast<int>(threadIdx.x) * 8;   // kBatch == kThreads * 8
        const int i0 = w0 - d0;                                     // child index of entry w0
        float x[8];
        bool p[8];
        bool any = false;
        if (w0 < d0 + deg) {
          win_load8(w0, x);
#pragma unroll
          for (int i = 0; i < 8; ++i) {
            const float sc = __fadd_rn(c.cum, __fsub_rn(x[i], lse));
            p[i] = (i0 + i >= 0) && (i0 + i < deg) && (sc >= thr_s || c.lo_tok + i0 + i == P.eos);
            any |= p[i];
          }
        } else {
#pragma unroll
          for (int i = 0; i < 8; ++i) p[i] = false;
        }
        if (__any_sync(0xFFFFFFFFu, any)) {
          uint64_t kv[8];
          uint32_t mask = 0;
#pragma unroll
          for (int i = 0; i < 8; ++i) {
            kv[i] = 0;
            if (p[i]) {
              kv[i] = child_key(c, c.lo_tok + i0 + i, i0 + i, x[i], lse, fb);
              if (kv[i] >= thr) mask |= 1u << i;
            }
          }
          warp_append_n<8>(mask, kv, S.keys, &S.v->cnt, kKeyCap, &S.v->overflow);
        }
        if (threadIdx.x == 0 && tau_g > S.v->thr_key) S.v->thr_key = tau_g;
        const int n_list = list_len_sync();
        if (base + kBatch < d0 + deg && n_list > kKeyCap - kBatch) {
          const Cut cut = shrink_to(P.k2);
          raise_tau(c.r, cut.floor_key());
        }
      }
    } else if (P.vstride > 1 && c.dense) {
      // a dense node of a strided shard: the shard's children of it sit in
      // local columns first_l .. last_l (tokens first_l * vstride + voff, ...)
      const int first_l = col_ceil(P, c.lo_tok);
      const int nloc = max(0, min(col_floor(P, c.lo_tok + deg - 1), P.VL - 1) - first_l + 1);
      for (int base = 0; base < nloc; base += kThreads) {
        const uint64_t thr = S.v->thr_key;
        const float thr_s = thr ? key_score(thr) : -kInf;
        const int tl = first_l + base + static_cast<int>(threadIdx.x);
        const int tok = tok_of(P, tl);
        bool pass = false;
        float x = 0.0f;
        if (base + static_cast<int>(threadIdx.x) < nloc) {
          x = (tl >= c.wlo && tl <= c.whi) ? win_load(tl - c.wlo) : load_logit(c, tl);
          pass = (__fadd_rn(c.cum, __fsub_rn(exact_y(c, x, tl), lse)) >= thr_s) || tok == P.eos;
        }
        uint64_t kv[1] = {0ull};
        uint32_t mask = 0;
        if (pass) {
          kv[0] = child_key(c, tok, tok - c.lo_tok, x, lse, fb);   // the key carries the child's index
          if (kv[0] >= thr) mask = 1u;
        }
        warp_append_n<1>(mask, kv, S.keys, &S.v->cnt, kKeyCap, &S.v->overflow);
        const int n_list = list_len_sync();
        if (base + kThreads < nloc && n_list > kKeyCap - kThreads) {
          const Cut cut = shrink_to(P.k2);
          raise_tau(c.r, cut.floor_key());
        }
      }
    } else {
      constexpr int kPer = kBatch / kThreads;
      for (int base = c0; base < c1; base += kBatch) {
        const int end = min(base + kBatch, c1);
        const uint64_t thr = S.v->thr_key;
        const float thr_s = thr ? key_score(thr) : -kInf;
        uint64_t tau_g = 0;
        if (threadIdx.x == 0 && end < c1) tau_g = *reinterpret_cast<volatile unsigned long long*>(P.tau + c.r);
        // issue every child-token load of the batch before using any of them
        int toks[kPer];
#pragma unroll
        for (int i = 0; i < kPer; ++i) {
          const int j = base + i * kThreads + static_cast<int>(threadIdx.x);
          toks[i] = (j >= end) ? -1
                  : (c.dense ? c.lo_tok + (j - c0)
                             : (deg <= kMetaSmall ? rec[kMToks + (j - c0)] : __ldg(P.child_tok + j)));
        }
        float xs[kPer];
        bool p[kPer];
        bool any = false;
#pragma unroll
        for (int i = 0; i < kPer; ++i) {
          const int tok = toks[i];
          p[i] = false;
          xs[i] = 0.0f;
          if (tok >= 0) {
            if (tok >= P.V) {
              atomicOr(P.err, GR_DEVERR_BAD_CHILD);
            } else {
              const int tl = col_of(P, tok);
              if (tl >= 0) {
                const float x = (tl >= c.wlo && tl <= c.whi) ? win_load(tl - c.wlo) : load_logit(c, tl);
                xs[i] = x;
                const float y = exact_y(c, x, tl);
                const float sc = __fadd_rn(c.cum, __fsub_rn(y, lse));
                p[i] = (sc >= thr_s) || tok == P.eos;
              }
            }
          }
          any |= p[i];
        }
        if (__any_sync(0xFFFFFFFFu, any)) {
          uint64_t kv[kPer];
          uint32_t mask = 0;
#pragma unroll
          for (int i = 0; i < kPer; ++i) {
            kv[i] = 0;
            if (p[i]) {
              kv[i] = child_key(c, toks[i], base + i * kThreads + static_cast<int>(threadIdx.x) - c0, xs[i], lse, fb);
              if (kv[i] >= thr) mask |= 1u << i;
            }
          }
          warp_append_n<kPer>(mask, kv, S.keys, &S.v->cnt, kKeyCap, &S.v->overflow);
        }
        if (threadIdx.x == 0 && tau_g > S.v->thr_key) S.v->thr_key = tau_g;
        const int n_list = list_len_sync();
        if (end < c1 && n_list > kKeyCap - kBatch) {
          const Cut cut = shrink_to(P.k2);
          raise_tau(c.r, cut.floor_key());
        }
      }
    }
    if (static_cast<int>(S.v->cnt) > P.k2) {
      const Cut cut = shrink_to(P.k2);
      raise_tau(c.r, cut.floor_key());
    }
  }

  // The largest log-prob-domain value below y that a column of this row can
  // hold.  A streamed row that dropped columns kept every column whose key
  // (value, then lower flat index) beats the dropped ones, so a dropped column
  // has the kept minimum value y_last (and a larger flat index than the kept
  // columns of that value) or a value at most value_below(y_last).  Raw 2-byte
  // logits step to the next lower value of their type; otherwise (f32 logits,
  // or processed values x / T) to the next lower float32.
  __device__ __forceinline__ float value_below(float y) const {
    if (!(y > -kInf)) return y;                      // -inf (nothing below) or NaN
    if constexpr (ES == 2) {
      if (P.mode != kModeProcessed) {
        uint32_t h;
        if constexpr (std::is_same_v<TL, __nv_bfloat16>) h = __float_as_uint(y) >> 16;
        else h = __half_as_ushort(__float2half_rn(y));
        const uint32_t sign = 0x8000u;
        h = ((h & 0x7FFFu) == 0u) ? (sign | 1u) : ((h & sign) ? h + 1u : h - 1u);
        if constexpr (std::is_same_v<TL, __nv_bfloat16>) return __uint_as_float(h << 16);
        else return __half2float(__ushort_as_half(static_cast<unsigned short>(h)));
      }
    }
    const uint32_t u = __float_as_uint(y);
    if ((u & 0x7FFFFFFFu) == 0u) return -__uint_as_float(1u);   // -0 / +0 -> the smallest negative
    return __uint_as_float((u & 0x80000000u) ? u + 1u : u - 1u);
  }

  // Exact top-k of the row's columns from global memory, keyed by score
  // (cum + (y - lse), EOS at -inf) or, with lp_only, by log-prob (y - lse):
  // for streamed rows whose dropped columns could tie the kept boundary after
  // rounding.  Keys beating a running bound (the k-th key of a k-subset, a
  // lower bound of the row's k-th) are appended in batches; the list is cut
  // back to k whenever the next batch might not fit.
  __device__ void rescan_row(const RowCtx& c, float lse, int k, bool lp_only) {
    const Smem S = smem_view(P);
    csync();
    if (threadIdx.x == 0) {
      S.v->cnt = 0;
      S.v->overflow = 0;
    }
    csync();
    constexpr int kMaxPer = kBatch / kThreads;
    // columns per thread per batch: a batch must fit beside the k kept keys
    const int per = max(1, min(kMaxPer, (kKeyCap - k) / kThreads));
    const int nb = per * kThreads;
    const uint32_t fb = static_cast<uint32_t>(c.b) * static_cast<uint32_t>(P.V);
    uint64_t thr = 0ull;
    for (int base = 0; base < P.VL; base += nb) {
      uint64_t kv[kMaxPer];
      uint32_t mask = 0;
#pragma unroll
      for (int i = 0; i < kMaxPer; ++i) {
        kv[i] = 0ull;
        const int tl = base + i * kThreads + static_cast<int>(threadIdx.x);
        if (i < per && tl < P.VL) {
          const float lp = __fsub_rn(exact_y(c, load_logit(c, tl), tl), lse);
          float sc = lp_only ? lp : __fadd_rn(c.cum, lp);
          const int tok = tok_of(P, tl);
          if (!lp_only && tok == P.eos) sc = -kInf;
          kv[i] = make_key(sc, fb + static_cast<uint32_t>(tok));
          if (kv[i] >= thr) mask |= 1u << i;
        }
      }
      warp_append_n<kMaxPer>(mask, kv, S.keys, &S.v->cnt, kKeyCap, &S.v->overflow);
      const int n_list = list_len_sync();
      if (base + nb < P.VL && n_list > kKeyCap - nb) thr = shrink_to(k).floor_key();
    }
    if (static_cast<int>(S.v->cnt) > k) shrink_to(k);
  }

  // Streamed rows: convert the kept value-keys (ord(y) | ~flat) into score keys.
  // A row that dropped columns is read again exactly when a dropped column
  // could score as high as the row's 2B-th candidate.
  __device__ void unconstrained_candidates(const RowCtx& c, float lse) {
    const Smem S = smem_view(P);
    // the kept set holds the row's best kk value-keys (all of them if nothing was discarded)
    if (static_cast<int>(S.v->cnt) > P.kk) {
      shrink_to(P.kk);
      if (threadIdx.x == 0) S.v->discard = 1;
      csync();
    }
    const bool discarded = S.v->discard != 0;
    float y_last = -kInf;
    if (discarded) y_last = key_score(min_key_of_list());
    const int n = min(static_cast<int>(S.v->cnt), kKeyCap);
    const uint32_t vb = static_cast<uint32_t>(c.b) * static_cast<uint32_t>(P.V);
    for (int i = threadIdx.x; i < n; i += kThreads) {
      const uint64_t k = S.keys[i];
      const uint32_t flat = key_flat(k);
      const int tok = static_cast<int>(flat - vb);
      float sc = __fadd_rn(c.cum, __fsub_rn(key_score(k), lse));
      if (tok == P.eos) sc = -kInf;
      S.keys[i] = make_key(sc, flat);
    }
    const int eos_l = (P.eos >= 0) ? col_of(P, P.eos) : -1;
    if (threadIdx.x == 0 && eos_l >= 0 && P.eos_score) {
      const int tl = eos_l;
      const float y = exact_y(c, load_logit(c, tl), tl);
      P.eos_score[c.row] = __fadd_rn(c.cum, __fsub_rn(y, lse));
    }
    csync();
    if (n > P.k2) {
      // the row's 2B-th key bounds the request (any 2B of its candidates do)
      const Cut cut = shrink_to(P.k2);
      if (P.K == 0) raise_tau(c.r, cut.floor_key());
    }
    if (discarded && n > 0) {
      // a dropped column scores at most s_below; equal to the 2B-th score, it
      // might precede it by flat index: take the row's exact top-2B instead
      const float s_below = __fadd_rn(c.cum, __fsub_rn(value_below(y_last), lse));
      const float s_kth = key_score(min_key_of_list());
      if (!(s_below < s_kth)) rescan_row(c, lse, P.k2, false);
    }
  }

  // Reference-literal rows: the beam's own top-K by log-prob (vLLM topk),
  // de-duplicated against the greedy token, then masked to the catalog.
  __device__ void literal_candidates(const RowCtx& c, float lse) {
    const Smem S = smem_view(P);
    if (static_cast<int>(S.v->cnt) > P.kk) {
      shrink_to(P.kk);
      if (threadIdx.x == 0) S.v->discard = 1;
      csync();
    }
    const bool discarded = S.v->discard != 0;
    const uint32_t vb = static_cast<uint32_t>(c.b) * static_cast<uint32_t>(P.V);
    // greedy (sampled) token: argmax of the penalised logits, lowest id on ties
    int sampled_tl = -1;
    if (c.pen_active) {
      // candidates: every kept non-penalised column (value = raw logit) and
      // every penalised column (value = its penalised logit from the table)
      const int n = min(static_cast<int>(S.v->cnt), kKeyCap);
      uint64_t best = 0;
      for (int i = threadIdx.x; i < n; i += kThreads) {
        const int tl = col_of(P, static_cast<int>(key_flat(S.keys[i]) - vb));
        if (flagged(c, tl)) continue;
        const uint64_t k = make_key(load_logit(c, tl), static_cast<uint32_t>(tl));
        best = k > best ? k : best;
      }
      const int nt = static_cast<int>(S.v->ntab);
      for (int j = threadIdx.x; j < nt; j += kThreads) {
        const uint64_t k = make_key(S.tab_xp[j], static_cast<uint32_t>(S.tab_tok[j]));
        best = k > best ? k : best;
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) {
        const uint64_t v = __shfl_xor_sync(0xFFFFFFFFu, best, o);
        best = v > best ? v : best;
      }
      if (threadIdx.x == 0) S.v->min_key = 0;
      csync();
      if (lane_id() == 0) atomicMax(reinterpret_cast<unsigned long long*>(&S.v->min_key), best);
      csync();
      sampled_tl = (S.v->min_key == 0) ? -1 : static_cast<int>(key_flat(S.v->min_key));
      csync();
    }
    // value keys -> log-prob keys (ties: lower token first)
    float y_last = -kInf;
    if (discarded) y_last = key_score(min_key_of_list());
    int n = min(static_cast<int>(S.v->cnt), kKeyCap);
    for (int i = threadIdx.x; i < n; i += kThreads) {
      const uint64_t k = S.keys[i];
      S.keys[i] = make_key(__fsub_rn(key_score(k), lse), key_flat(k));
    }
    csync();
    const int K = min(P.K, n);
    if (n > K) shrink_to(K);
    n = min(static_cast<int>(S.v->cnt), kKeyCap);
    uint64_t kth = (n > 0) ? min_key_of_list() : 0ull;
    if (discarded && n > 0 && !(__fsub_rn(value_below(y_last), lse) < key_score(kth))) {
      // a dropped column might tie the K-th log-prob and precede it by token:
      // the row's exact top-K instead
      rescan_row(c, lse, P.K, true);
      n = min(static_cast<int>(S.v->cnt), kKeyCap);
      kth = (n > 0) ? min_key_of_list() : 0ull;
    }
    // dedup against the sampled token (vllm_gr/logprobs.py:47-52)
    if (sampled_tl >= 0) {
      const uint32_t sflat = vb + static_cast<uint32_t>(tok_of(P, sampled_tl));
      if (threadIdx.x == 0) S.v->last = 0;
      csync();
      for (int i = threadIdx.x; i < n; i += kThreads)
        if (key_flat(S.keys[i]) == sflat) S.v->last = 1;
      csync();
      if (S.v->last == 0 && n > 0) {
        // replace the K-th (smallest) entry by the sampled token
        const float ys = exact_y(c, load_logit(c, sampled_tl), sampled_tl);
        const uint64_t sk = make_key(__fsub_rn(ys, lse), sflat);
        for (int i = threadIdx.x; i < n; i += kThreads)
          if (S.keys[i] == kth) S.keys[i] = sk;
      }
      csync();
    }
    // catalog mask, cum add, EOS (serving_engine.py:504-506, 511, 541-562)
    for (int i = threadIdx.x; i < n; i += kThreads) {
      const uint64_t k = S.keys[i];
      const uint32_t flat = key_flat(k);
      const int tok = static_cast<int>(flat - vb);
      bool allowed = true;
      if (c.node >= 0) {
        int lo = c.c0, hi = c.c1;
        while (lo < hi) {
          const int mid = (lo + hi) >> 1;
          if (P.child_tok[mid] < tok) lo = mid + 1; else hi = mid;
        }
        allowed = (lo < c.c1) && (P.child_tok[lo] == tok);
      } else if (c.node == GR_NODE_DEAD) {
        allowed = false;
      }
      float sc = allowed ? __fadd_rn(c.cum, key_score(k)) : -kInf;
      if (tok == P.eos) {
        if (P.eos_score) P.eos_score[c.row] = sc;
        sc = -kInf;
      }
      S.keys[i] = make_key(sc, flat);
    }
    csync();
    if (n > P.k2) shrink_to(P.k2);
  }

  // Write the row's keys that beat the request threshold into the row's own
  // slot of the candidate buffer (no atomics; the merge kernel gathers them).
  __device__ void emit(const RowCtx& c, bool refilter) {
    const Smem S = smem_view(P);
    int n;
    if (refilter) {
      if (threadIdx.x == 0) {
        const uint64_t t = S.v->tau_pref;       // read at row start; a stale bound is still valid
        if (t > S.v->thr_key) S.v->thr_key = t;
      }
      csync();
      const uint64_t thr = S.v->thr_key;
      n = min(static_cast<int>(S.v->cnt), kKeyCap);
      if (thr > 0 && n > 0) n = static_cast<int>(cta_compact(S.keys, n, Cut{thr, 0}, &S.v->cnt));
    } else {
      n = min(static_cast<int>(S.v->cnt), kKeyCap);
    }
    if (n > P.k2) {                     // cannot happen: every path selects at most 2B
      if (threadIdx.x == 0) atomicOr(P.err, GR_DEVERR_OVERFLOW);
      n = P.k2;
    }
    // append to the request's candidate list (one reservation per row); the
    // merge reads it right after this kernel: keep it in L2 ahead of the stream
    if (threadIdx.x == 0) S.v->base = (n > 0) ? atomicAdd(P.rowcnt + static_cast<size_t>(c.r) * P.NB, static_cast<unsigned>(n)) : 0u;
    csync();
    unsigned long long* dst = P.buf + static_cast<size_t>(c.r) * P.NB * static_cast<size_t>(P.k2) + S.v->base;
    const uint64_t keep = l2_policy_evict_last();
    for (int i = threadIdx.x; i < n; i += kThreads) st_keep_u64(dst + i, S.keys[i], keep);
    if (P.req_hist && n > 0) raise_tau_from_histogram(c, n);
  }

  // Add this row's emitted keys to its request's score histogram and raise the
  // request bound to the first bin where the count from the top reaches 2B.
  __device__ void raise_tau_from_histogram(const RowCtx& c, int n) {
    const Smem S = smem_view(P);
    static_assert(kKeyCap / 2 * 2 >= kReqHistBins, "local histogram fits in the key list's upper half");
    uint32_t* lh = reinterpret_cast<uint32_t*>(S.keys + kKeyCap / 2);   // keys use [0, 2B <= kKeyCap/2)
    const float ref = __int_as_float(rec[kMRef]);
    for (int i = threadIdx.x; i < kReqHistBins; i += kThreads) lh[i] = 0u;
    csync();
    for (int i = threadIdx.x; i < n; i += kThreads) {
      const float d = (ref - key_score(S.keys[i])) * kReqHistScale;
      // above the reference -> bin 0; NaN, -inf and far below -> the catch-all last bin
      const int bin = (d < 0.0f) ? 0 : ((d >= 0.0f && d < kReqHistBins - 1) ? static_cast<int>(d) : kReqHistBins - 1);
      atomicAdd(&lh[bin], 1u);
    }
    csync();
    unsigned int* gh = P.req_hist + static_cast<size_t>(c.r) * kReqHistBins;
    constexpr int kPer = kReqHistBins / kThreads;
    uint32_t cnt[kPer];
    uint32_t mine = 0;
#pragma unroll
    for (int q = 0; q < kPer; ++q) {
      const int bin = threadIdx.x * kPer + q;
      const uint32_t add = lh[bin];
      cnt[q] = add ? atomicAdd(gh + bin, add) + add : __ldcg(gh + bin);
      if (bin == kReqHistBins - 1) cnt[q] = 0;   // the catch-all bin bounds nothing
      mine += cnt[q];
    }
    // exclusive prefix over threads (bins in order: best first)
    const int lane = lane_id(), warp = warp_id();
    uint32_t inc = mine;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const uint32_t v = __shfl_up_sync(0xFFFFFFFFu, inc, o);
      if (lane >= o) inc += v;
    }
    float* wsum = S.red_m;   // kWarps words, free outside the row-end normaliser
    if (lane == 31) wsum[warp] = __uint_as_float(inc);
    csync();
    uint32_t before = inc - mine;
    for (int w = 0; w < warp; ++w) before += __float_as_uint(wsum[w]);
    if (before < static_cast<uint32_t>(P.k2) && before + mine >= static_cast<uint32_t>(P.k2)) {
      uint32_t acc = before;
#pragma unroll
      for (int q = 0; q < kPer; ++q) {
        acc += cnt[q];
        if (acc >= static_cast<uint32_t>(P.k2)) {
          // 2B emitted keys score at least the lower edge of this bin (one more
          // bin of margin covers the rounding of the bin arithmetic)
          const float edge = ref - static_cast<float>(threadIdx.x * kPer + q + 2) / kReqHistScale;
          const uint64_t cand = static_cast<uint64_t>(f32_to_ord(__fadd_rn(edge, 0.0f))) << 32;
          atomicMax(P.tau + c.r, static_cast<unsigned long long>(cand));
          break;
        }
      }
    }
    csync();
  }
};

// Row context from the row's metadata record (c.row, c.r, c.b already set).
template <typename TL>
__device__ __forceinline__ void fill_row_ctx(const Params& P, const int* rec, RowCtx& c) {
  c.node = rec[kMNode];
  c.stream = (P.K > 0) || (c.node == GR_NODE_UNCONSTRAINED);
  c.constrained = !c.stream && c.node >= 0;
  c.c0 = rec[kMC0];
  c.c1 = rec[kMC1];
  c.wlo = 1;
  c.whi = 0;
  c.lo_tok = 0;
  c.dense = false;
  if (c.constrained && c.c1 > c.c0) {
    const int lt = rec[kMLo], ht = rec[kMHi];
    c.lo_tok = lt;
    c.dense = (ht - lt + 1) == (c.c1 - c.c0);
    const int lo = col_ceil(P, lt);
    const int hi = min(col_floor(P, ht), P.VL - 1);
    if (lo <= hi) {
      c.wlo = lo & ~7;                 // window index 0 = an 8-aligned column
      c.whi = min(hi, c.wlo + Step<TL>::kWinTok - 1);
    }
  }
  c.cum = __int_as_float(rec[kMCum]);
  c.teff = __int_as_float(rec[kMTeff]);
  c.rteff = __int_as_float(rec[kMRteff]);
  // penalties matter for processed log-probs and for the per-beam top-K's greedy token
  const bool pen_used = P.pen && P.T > 0 &&
                        (P.partial_only ? P.mode == kModeProcessed : (P.mode == kModeProcessed || P.K > 0));
  c.rep = (pen_used && P.rep) ? P.rep[c.r] : 1.0f;
  c.pres = (pen_used && P.pres) ? P.pres[c.r] : 0.0f;
  c.freq = (pen_used && P.freq) ? P.freq[c.r] : 0.0f;
  c.pen_active = pen_used && !(c.rep == 1.0f && c.pres == 0.0f && c.freq == 0.0f);
  if (P.partial_only) {
    // vocab-sharded phase 1: only the normaliser of the local columns
    c.stream = false;
    c.constrained = false;
  }
  c.excl = c.pen_active && P.mode == kModeProcessed;
}

// Add the fast-path accumulators (relative to the same reference max) into s.
__device__ __forceinline__ void fold(uint64_t& a0, uint64_t& a1, float& s) {
  float q0, q1, q2, q3;
  unpack2(a0, q0, q1);
  unpack2(a1, q2, q3);
  s += (q0 + q1) + (q2 + q3);
  a0 = pack2(0.0f, 0.0f);
  a1 = pack2(0.0f, 0.0f);
}

// Lazily normalised sum of exp over one chunk share of a thread (fast path):
// s += sum 2^(x*a - m*log2e) with the running reference m left unchanged unless
// the partial sum overflows (then the exact per-vector path recomputes it).
template <typename TL>
struct FastSum;

// Word groups of a 16-byte vector (of 4) whose exponentials use the FMA-pipe
// polynomial instead of the MUFU unit (2-byte logits only, where the MUFU rate
// is the tighter limit: 8 exponentials per 16 bytes).
#ifndef GR_POLY_EXP_GROUPS
#define GR_POLY_EXP_GROUPS 0
#endif

__device__ __forceinline__ uint64_t exp2_pair(uint64_t t2, bool poly) {
  if (poly) return poly_exp2x2(t2);
  float t0, t1;
  unpack2(t2, t0, t1);
  return pack2(fast_exp2(t0), fast_exp2(t1));
}

template <>
struct FastSum<__nv_bfloat16> {
  static constexpr int kWords = 4;   // 32-bit words per 16-byte vector
  __device__ static __forceinline__ void add(const uint4& v, uint64_t A2, uint64_t C2, uint64_t& p0, uint64_t& p1) {
    const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const uint64_t x2 = pack2(__uint_as_float(w[i] << 16), __uint_as_float(w[i] & 0xFFFF0000u));
      const uint64_t e2 = exp2_pair(ffma2(x2, A2, C2), i >= 4 - GR_POLY_EXP_GROUPS);
      if (i & 1) p1 = fadd2(p1, e2); else p0 = fadd2(p0, e2);
    }
  }
};

template <>
struct FastSum<__half> {
  __device__ static __forceinline__ void add(const uint4& v, uint64_t A2, uint64_t C2, uint64_t& p0, uint64_t& p1) {
    const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&w[i]));
      const uint64_t e2 = exp2_pair(ffma2(pack2(f.x, f.y), A2, C2), i >= 4 - GR_POLY_EXP_GROUPS);
      if (i & 1) p1 = fadd2(p1, e2); else p0 = fadd2(p0, e2);
    }
  }
};

template <>
struct FastSum<float> {
  __device__ static __forceinline__ void add(const uint4& v, uint64_t A2, uint64_t C2, uint64_t& p0, uint64_t& p1) {
    float t0, t1, t2, t3;
    unpack2(ffma2(pack2(__uint_as_float(v.x), __uint_as_float(v.y)), A2, C2), t0, t1);
    unpack2(ffma2(pack2(__uint_as_float(v.z), __uint_as_float(v.w)), A2, C2), t2, t3);
    p0 = fadd2(p0, pack2(fast_exp2(t0), fast_exp2(t1)));
    p1 = fadd2(p1, pack2(fast_exp2(t2), fast_exp2(t3)));
  }
};

// Producer warp, lane 0: fill the ring (stages of SB bytes at `ring`) with the
// CTA's (row, chunk) sequence.
// Vocab-sharded phase 2 (the rows' lse given): only rows without a node need
// their stream (their candidates are streamed values); the others read their
// child window directly.  Producer and consumers decide it from the same
// node, so they agree on every row's stage count.
__device__ __forceinline__ bool stream_skipped(const Params& P, int node) {
  return P.lse_in != nullptr && P.K == 0 && node != GR_NODE_UNCONSTRAINED;
}

template <int ES, int SB = kStageBytes>
__device__ __forceinline__ void produce(const Params& P, int my_n, unsigned char* ring) {
  const Smem S = smem_view(P);
  const uint64_t pol = l2_policy_evict_first();
  int stage = 0;
  uint32_t round = 0;
  long long fills = 0;
  for (int it = 0; it < (P.stall_copies ? 0 : my_n); ++it) {
    const int row = row_of_iter(P, it);
    const Geom g = row_geom<ES, SB>(P, row);
    const int nch = stream_skipped(P, __ldg(P.meta + static_cast<size_t>(row) * kMetaWords + kMNode)) ? 0 : g.nchunks;
    for (int ch = 0; ch < nch; ++ch) {
      if (fills >= P.stages) {
        if (!mbar_wait_bounded(&S.empty[stage], (round - 1u) & 1u, &S.v->abort)) {
          if (!S.v->abort) atomicOr(P.err, GR_DEVERR_TIMEOUT);
          S.v->abort = 1;
          goto done;
        }
      }
      {
        const long long off = static_cast<long long>(ch) * SB;
        const uint32_t bytes = static_cast<uint32_t>(min(static_cast<long long>(SB), g.body_bytes - off));
        fence_proxy_async_smem();
        mbar_arrive_expect_tx(&S.full[stage], bytes);
        bulk_copy_g2s(ring + static_cast<size_t>(stage) * SB, g.body + off, bytes, &S.full[stage], pol);
      }
      ++fills;
      if (++stage == P.stages) {
        stage = 0;
        ++round;
      }
    }
  }
done:
  S.v->issued = fills;
  __threadfence_block();
  S.v->producer_done = 1;
}

// One thread per row: node -> CSR range -> child-token bounds (and, for small
// nodes, every child token).
__global__ void __launch_bounds__(256) row_meta_kernel(const __grid_constant__ Params P) {
  pdl_trigger();   // the step kernel may start its prologue; it waits for this grid before reading
  // launched early as well (behind the previous step's merge, which reads this
  // workspace): nothing is read or written before that grid is complete
  pdl_wait();
  const int row = blockIdx.x * blockDim.x + threadIdx.x;
  if (row >= P.R * P.NB) return;
  if (row % P.NB == 0) {
    P.tau[row / P.NB] = 0ull;     // the request's running bound starts empty
    P.rowcnt[row] = 0u;           // and its candidate list
  }
  // GR_STEP_CLEAR_ERR: the error word starts at 0.  Nothing else in this grid
  // writes it then (a bad node goes into its record, reported by the merge),
  // and every later kernel writes it only after waiting for this grid.
  if (P.clear_err && row == 0) *P.err = 0;
  if (row == 0) *P.row_counter = 0u;
  int w[kMetaWords];
#pragma unroll
  for (int i = 0; i < kMetaWords; ++i) w[i] = 0;
  int node = P.node[row];
  if (node < GR_NODE_DEAD || node >= P.N) {
    if (P.clear_err) w[kMBad] = 1;
    else atomicOr(P.err, GR_DEVERR_BAD_NODE);
    node = GR_NODE_DEAD;
  }
  const int r = row / P.NB;
  const float teff = (P.mode == kModeProcessed) ? eff_temperature(P, r) : 1.0f;
  w[kMNode] = node;
  w[kMCum] = __float_as_int(P.cum[row]);
  w[kMTeff] = __float_as_int(teff);
  w[kMRteff] = __float_as_int(__frcp_rn(teff));
  w[kMRow] = row;
  w[kMR] = r;
  w[kMB] = row - r * P.NB;
  w[kMRef] = __float_as_int(P.cum[static_cast<size_t>(r) * P.NB]);
  if (P.req_hist) {
    // this row's share of its request's score histogram, zeroed for the step
    const int b = row - r * P.NB;
    for (int i = b; i < kReqHistBins; i += P.NB) P.req_hist[static_cast<size_t>(r) * kReqHistBins + i] = 0u;
  }
  if (node >= 0) {
    const int c0 = static_cast<int>(P.row_ptr[node]);
    const int c1 = static_cast<int>(P.row_ptr[node + 1]);
    w[kMC0] = c0;
    w[kMC1] = c1;
    if (c1 > c0) {
      w[kMLo] = P.child_tok[c0];
      w[kMHi] = P.child_tok[c1 - 1];
      if (c1 - c0 <= kMetaSmall)
        for (int j = 0; j < c1 - c0; ++j) w[kMToks + j] = P.child_tok[c0 + j];
    }
  }
  int4* dst = reinterpret_cast<int4*>(P.meta + static_cast<size_t>(row) * kMetaWords);
  const uint64_t keep = l2_policy_evict_last();   // read by the step and merge kernels
#pragma unroll
  for (int i = 0; i < kMetaWords / 4; ++i) st_keep_v4(dst + i, make_int4(w[4 * i], w[4 * i + 1], w[4 * i + 2], w[4 * i + 3]), keep);
}

template <typename TL>
__global__ void __launch_bounds__(kBlock, 2) fused_step_kernel(const __grid_constant__ Params P) {
  const Smem S = smem_view(P);
  Step<TL> st(P);
  using Tr = LogitTraits<TL>;
  constexpr int ES = sizeof(TL);
  constexpr int EPV = Tr::kPerVec;
  constexpr int kChunkElems = kStageBytes / ES;
  constexpr int kChunkVecs = kStageBytes / 16;

  const int tid = threadIdx.x, lane = lane_id(), warp = warp_id();
  const int total = P.R * P.NB;
  const int my_n = (static_cast<int>(blockIdx.x) < total) ? (total - 1 - static_cast<int>(blockIdx.x)) / static_cast<int>(gridDim.x) + 1 : 0;

  if (tid == 0) {
    for (int s = 0; s < P.stages; ++s) {
      mbar_init(&S.full[s], 1);
      mbar_init(&S.empty[s], kWarps);
    }
    fence_mbar_init();
    S.v->abort = 0;
    S.v->producer_done = 0;
    S.v->issued = 0;
  }
  if (P.pen)
    for (int i = tid; i < P.bm_words; i += kBlock) S.bitmap[i] = 0u;
  GR_PROF_INIT();
  pdl_wait();        // row metadata and the zeroed bounds come from the previous kernel
  pdl_trigger();
  __syncthreads();   // the only CTA-wide barrier: consumers use csync() from here on

  if (warp == kWarps) {
    if (lane == 0) produce<ES>(P, my_n, S.ring);
    return;
  }

  int cstage = 0;
  uint32_t cphase = 0;
  long long consumed = 0;
  int meta_word = 0;                 // word tid (< kMetaWords) of the next row's metadata record
  GR_PROF_T(t_kernel);
  for (int it = 0; it < my_n; ++it) {
    // ------------------------------------------------------------ row setup
    GR_PROF_CNT(10);
    GR_PROF_T(t_row);
    RowCtx c;
    c.row = row_of_iter(P, it);
    c.r = c.row / P.NB;
    c.b = c.row - c.r * P.NB;
    // the row's metadata record: word tid was prefetched during the previous row
    if (it == 0 && tid < kMetaWords) meta_word = __ldcg(P.meta + static_cast<size_t>(c.row) * kMetaWords + tid);
    if (tid < kMetaWords) S.v->meta[tid] = meta_word;
    csync();
    if (tid < kMetaWords && it + 1 < my_n)
      meta_word = __ldcg(P.meta + static_cast<size_t>(row_of_iter(P, it + 1)) * kMetaWords + tid);
    fill_row_ctx<TL>(P, S.v->meta, c);
    st.rec = S.v->meta;
    const bool fast_ok = !c.stream && !c.excl;

    if (tid == 0) {
      S.v->cnt = 0;
      S.v->ntab = 0;
      S.v->overflow = 0;
      S.v->discard = 0;
      S.v->thr_key = 0ull;
      S.v->thr_y = -kInf;
      if (P.eos_score && !P.partial_only) P.eos_score[c.row] = __int_as_float(0x7FC00000);
    }
    if (tid < kWarps) S.v->lse_w[tid] = -kInf;
    csync();
    if (c.pen_active) {
      const int* h = P.hist + static_cast<size_t>(c.row) * P.T;
      for (int t = tid; t < P.T; t += kThreads) {
        const int tok = h[t];
        const int tl = (tok >= 0) ? col_of(P, tok) : -1;
        if (tl >= 0) {
          const uint32_t bit = 1u << (tl & 31);
          const uint32_t old = atomicOr(&S.bitmap[tl >> 5], bit);
          if (!(old & bit)) {
            int cnt = 0;
            for (int j = 0; j < P.T; ++j) cnt += (h[j] == tok);
            const float xp = penalise(st.load_logit(c, tl), cnt, c.rep, c.pres, c.freq);
            const uint32_t idx = atomicAdd(&S.v->ntab, 1u);
            S.tab_tok[idx] = tl;
            S.tab_xp[idx] = xp;
            S.tab_y[idx] = (P.mode == kModeProcessed) ? ((c.teff == 1.0f) ? xp : __fdiv_rn(xp, c.teff)) : xp;
          }
        }
      }
      csync();
    }

    // the request's running threshold: loaded now, used after the stream
    uint64_t tau_pref = 0;
    if (tid == 0 && !P.partial_only) tau_pref = *reinterpret_cast<volatile unsigned long long*>(P.tau + c.r);

    float m = -kInf, s = 0.0f;
    float thr_y = -kInf;
    uint64_t thr_key = 0ull;
    // streamed top-2B rows: the request bound as read one chunk earlier
    const bool bounded = c.stream && P.K == 0 && !P.partial_only;
    uint64_t tau_seen = bounded ? *reinterpret_cast<volatile unsigned long long*>(P.tau + c.r) : 0ull;
    const Geom g = row_geom<ES>(P, c.row);
    // whole-vector window copies need vectors that start on window-vector boundaries
    const bool win_vec_ok = (g.head % EPV) == 0;
    // fast-path scale: exp(y - m) = 2^(x * a - m * log2e) with y = x (raw) or x / T
    const float a = kLog2e * ((P.mode == kModeProcessed) ? c.rteff : 1.0f);
    uint64_t sacc0 = pack2(0.0f, 0.0f), sacc1 = pack2(0.0f, 0.0f);

    // ------------------------------------------------------- head / tail scalars
    {
      const int nh = g.head, nt = P.VL - g.tail_start;
      const int ns = nh + nt;
      for (int ib = warp * 32; ib < ns; ib += kThreads) {
        const int i = ib + lane;
        const bool valid = i < ns;
        const int tl = valid ? ((i < nh) ? i : g.tail_start + (i - nh)) : 0;
        float x[1];
        x[0] = valid ? st.load_logit(c, tl) : -kInf;
        st.template process<1>(c, x, tl, valid, m, s, thr_y, thr_key);
      }
    }
    // vocab-sharded phase 2: no stream for rows with a node; their window's
    // body columns are read here (the head and tail columns came just above)
    const int nch = stream_skipped(P, c.node) ? 0 : g.nchunks;
    if (nch == 0 && g.nchunks > 0 && c.constrained) {
      const int lo = max(c.wlo, g.head), hi = min(c.whi, g.tail_start - 1);
      for (int tl = lo + tid; tl <= hi; tl += kThreads) st.win_store(tl - c.wlo, st.load_logit(c, tl));
      csync();
    }
    // list length after the last complete append round, and the CTA's lse
    // bound (bounded rows)
    uint32_t cnt_prev = 0;
    float row_L = -kInf;
    if (bounded) {
      cnt_prev = static_cast<uint32_t>(st.list_len_sync());
    }
    // shrink the row's list back to its best kk keys; the kk-th bounds the rest of the row
    auto shrink_row = [&]() {
      const Cut cut = st.shrink_to(P.kk);
      if (tid == 0) {
        S.v->discard = 1;
        S.v->thr_key = cut.floor_key();
        const float ty = key_score(cut.floor_key());
        S.v->thr_y = ty - fabsf(ty) * 2.0e-6f - 1e-30f;
      }
      csync();
      thr_key = S.v->thr_key;
      thr_y = S.v->thr_y;
    };
    const uint32_t shrink_at = max(static_cast<uint32_t>(kKeyCap - 1024),
                                   static_cast<uint32_t>(P.kk + (kKeyCap - P.kk) / 2));

    // ------------------------------------------------------------ body chunks
    GR_PROF_ADD(5, t_row);
    GR_PROF_T(t_stream);
    for (int ch = 0; ch < nch; ++ch) {
      GR_PROF_T(t_wait);
      if (!mbar_wait_bounded(&S.full[cstage], cphase, &S.v->abort)) {
        if (!S.v->abort) atomicOr(P.err, GR_DEVERR_TIMEOUT);
        S.v->abort = 1;
      }
      GR_PROF_ADD(1, t_wait);
      const long long off = static_cast<long long>(ch) * kStageBytes;
      const int bytes = static_cast<int>(min(static_cast<long long>(kStageBytes), g.body_bytes - off));
      const int nvec = bytes >> 4;
      const uint4* sv = reinterpret_cast<const uint4*>(S.ring + static_cast<size_t>(cstage) * kStageBytes);
      const int tbase = g.head + ch * kChunkElems;
      const bool in_window = c.constrained && tbase + kChunkElems > c.wlo && tbase <= c.whi;
      if (fast_ok && (!in_window || win_vec_ok)) {
        // fast path: kVecPerThread 16-byte vectors per thread, packed f32x2 math
        constexpr int kVecPerThread = kChunkVecs / kThreads;
        static_assert(kChunkVecs % kThreads == 0, "whole vectors per thread per stage");
        uint4 vv[kVecPerThread];
#pragma unroll
        for (int j = 0; j < kVecPerThread; ++j)
          vv[j] = (tid + j * kThreads < nvec) ? sv[tid + j * kThreads] : make_uint4(0, 0, 0, 0);
        if (in_window) {
          // keep the raw vectors that fall in the row's child window (vector aligned)
          uint4* wv = reinterpret_cast<uint4*>(st.win());
#pragma unroll
          for (int j = 0; j < kVecPerThread; ++j) {
            const int tb = tbase + (tid + j * kThreads) * EPV;
            if (tid + j * kThreads < nvec && tb + EPV > c.wlo && tb <= c.whi) wv[(tb - c.wlo) / EPV] = vv[j];
          }
        }
        if (m == -kInf) {
          // seed the running reference with this thread's own maximum (any element works)
          float mx = -kInf;
#pragma unroll
          for (int j = 0; j < kVecPerThread; ++j) {
            if (tid + j * kThreads < nvec) {
              float x[EPV];
              Tr::unpack(vv[j], x);
#pragma unroll
              for (int i = 0; i < EPV; ++i) mx = fmaxf(mx, x[i]);
            }
          }
          m = (P.mode == kModeProcessed) ? mx * c.rteff : mx;
        }
        const float cm = -m * kLog2e;
        const uint64_t A2 = pack2(a, a), C2 = pack2(cm, cm);
        uint64_t p0 = pack2(0.0f, 0.0f), p1 = pack2(0.0f, 0.0f);
#pragma unroll
        for (int j = 0; j < kVecPerThread; ++j)
          if (tid + j * kThreads < nvec) FastSum<TL>::add(vv[j], A2, C2, p0, p1);
        float q0, q1, q2, q3;
        unpack2(p0, q0, q1);
        unpack2(p1, q2, q3);
        const float tot = (q0 + q1) + (q2 + q3);
        if (tot <= 1.0e30f) {
          sacc0 = fadd2(sacc0, p0);
          sacc1 = fadd2(sacc1, p1);
        } else {
          // first chunk of the row, a large partial sum or non-finite input:
          // fold the fast accumulators (same reference m) and take the exact path
          fold(sacc0, sacc1, s);
#pragma unroll
          for (int j = 0; j < kVecPerThread; ++j) {
            if (tid + j * kThreads < nvec) {
              float x[EPV];
              Tr::unpack(vv[j], x);
              float y[EPV];
#pragma unroll
              for (int i = 0; i < EPV; ++i) y[i] = (P.mode == kModeProcessed) ? x[i] * c.rteff : x[i];
              st.template lse_update<EPV>(y, m, s);
            }
          }
        }
      } else if (bounded) {
        // streamed top-2B row: the exponential sum of the whole stage first, then
        // a candidate pass against the request bound through a lower bound of the
        // row's lse; survivors get list slots with one reservation per warp and
        // one CTA barrier per stage
        constexpr int kVecPerThread = kChunkVecs / kThreads;
        const float y_scale = (P.mode == kModeProcessed) ? c.rteff : 1.0f;
        const uint64_t tau_use = tau_seen;
        tau_seen = *reinterpret_cast<volatile unsigned long long*>(P.tau + c.r);
        uint4 vv[kVecPerThread];
        uint32_t flv[kVecPerThread];
#pragma unroll
        for (int j = 0; j < kVecPerThread; ++j) {
          const int v = tid + j * kThreads;
          vv[j] = (v < nvec) ? sv[v] : make_uint4(0, 0, 0, 0);
          flv[j] = 0;
          if (c.excl && v < nvec) {
            // penalised columns take their exact values at the row end
            const int tb = tbase + v * EPV;
            const int w = tb >> 5, sh = tb & 31;
            uint64_t bits = S.bitmap[w];
            if (w + 1 < P.bm_words) bits |= static_cast<uint64_t>(S.bitmap[w + 1]) << 32;
            flv[j] = static_cast<uint32_t>(bits >> sh) & ((1u << EPV) - 1u);
            if (flv[j]) Tr::mask_neg_inf(vv[j], flv[j]);
          }
        }
        if (m == -kInf) {
          float mx = -kInf;
#pragma unroll
          for (int j = 0; j < kVecPerThread; ++j) {
            if (tid + j * kThreads < nvec) {
              float x[EPV];
              Tr::unpack(vv[j], x);
#pragma unroll
              for (int i = 0; i < EPV; ++i) mx = fmaxf(mx, x[i]);
            }
          }
          m = (P.mode == kModeProcessed) ? mx * c.rteff : mx;
        }
        {
          const float cm = -m * kLog2e;
          const uint64_t A2 = pack2(a, a), C2 = pack2(cm, cm);
          uint64_t p0 = pack2(0.0f, 0.0f), p1 = pack2(0.0f, 0.0f);
#pragma unroll
          for (int j = 0; j < kVecPerThread; ++j)
            if (tid + j * kThreads < nvec) FastSum<TL>::add(vv[j], A2, C2, p0, p1);
          float q0, q1, q2, q3;
          unpack2(p0, q0, q1);
          unpack2(p1, q2, q3);
          const float tot = (q0 + q1) + (q2 + q3);
          if (tot <= 1.0e30f) {
            s += tot;
          } else {
#pragma unroll
            for (int j = 0; j < kVecPerThread; ++j) {
              if (tid + j * kThreads < nvec) {
                float x[EPV];
                Tr::unpack(vv[j], x);
                float y[EPV];
#pragma unroll
                for (int i = 0; i < EPV; ++i) y[i] = (P.mode == kModeProcessed) ? x[i] * c.rteff : x[i];
                st.template lse_update<EPV>(y, m, s);
              }
            }
          }
        }
        // the CTA's lse bound: every stage at the row start, then every fourth
        // (it grows by log(n / (n - 1)) per stage; a stale one is still a bound)
        if (ch < 4 || (ch & 3) == 0) row_L = st.cta_lse_bound(m, s, S.v->lse_w);
        const float floor_y = st.tau_floor(c, tau_use, row_L);
        const float thr_e = fmaxf(thr_y, floor_y);
        // survivors: bit j * EPV + i for element i of vector j
        uint32_t pm = 0;
#pragma unroll
        for (int j = 0; j < kVecPerThread; ++j) {
          if (tid + j * kThreads < nvec) {
            float x[EPV];
            Tr::unpack(vv[j], x);
            float vmax = x[0];
#pragma unroll
            for (int i = 1; i < EPV; ++i) vmax = fmaxf(vmax, x[i]);
            if (vmax * y_scale >= thr_e) {
#pragma unroll
              for (int i = 0; i < EPV; ++i)
                if (!((flv[j] >> i) & 1u) && x[i] * y_scale >= thr_e) pm |= 1u << (j * EPV + i);
            }
          }
        }
        const uint32_t cl = static_cast<uint32_t>(__popc(pm));
        uint32_t inc = 0, base = 0;
        if (__any_sync(0xFFFFFFFFu, cl != 0)) {
          inc = cl;
#pragma unroll
          for (int o = 1; o < 32; o <<= 1) {
            const uint32_t t = __shfl_up_sync(0xFFFFFFFFu, inc, o);
            if (lane >= o) inc += t;
          }
          const uint32_t wtot = __shfl_sync(0xFFFFFFFFu, inc, 31);
          if (lane == 31) base = atomicAdd(&S.v->cnt, wtot);
          base = __shfl_sync(0xFFFFFFFFu, base, 31);
        }
        const uint32_t cnt_now = static_cast<uint32_t>(st.list_len_sync());
        GR_PROF_VAL(12, cnt_now - cnt_prev);
        GR_PROF_VAL(14, floor_y > -kInf ? 1 : 0);
        GR_PROF_CNT(15);
        if (cnt_now <= static_cast<uint32_t>(kKeyCap)) {
          if (cl) {
            const unsigned char* stage_p = S.ring + static_cast<size_t>(cstage) * kStageBytes;
            const uint32_t fbase = static_cast<uint32_t>(c.b) * static_cast<uint32_t>(P.V) +
                                   static_cast<uint32_t>(tok_of(P, tbase));
            uint32_t pos = base + inc - cl;
            uint32_t mk = pm;
            while (mk) {
              const int e = __ffs(mk) - 1;
              mk &= mk - 1u;
              const int col = (tid + (e / EPV) * kThreads) * EPV + (e % EPV);
              const float x = Tr::load_s(stage_p, col);
              const float ye = (P.mode == kModeProcessed && c.teff != 1.0f) ? __fdiv_rn(x, c.teff) : x;
              S.keys[pos++] = make_key(ye, fbase + static_cast<uint32_t>(col * P.vstride));
            }
          }
          cnt_prev = cnt_now;
        } else {
          // the reservations do not fit: undo them and append this stage in
          // sub-batches with capacity checks (the sums are already in m, s)
          GR_PROF_CNT(13);
          csync();
          if (tid == 0) S.v->cnt = cnt_prev;
          csync();
          for (int sb = 0; sb < nvec; sb += P.sub_vecs) {
            // room for a whole sub-batch first (the list may hold up to shrink_at keys)
            if (st.list_len_sync() > kKeyCap - P.sub_vecs * EPV) shrink_row();
            const int send = min(nvec, sb + P.sub_vecs);
            for (int vb = sb + warp * 32; vb < send; vb += kThreads) {
              const int v = vb + lane;
              const bool valid = v < send;
              float x[EPV];
              if (valid) {
                Tr::unpack(sv[v], x);
              } else {
#pragma unroll
                for (int i = 0; i < EPV; ++i) x[i] = -kInf;
              }
              st.template process<EPV>(c, x, tbase + v * EPV, valid, m, s, thr_y, thr_key, floor_y, false);
            }
          }
          cnt_prev = static_cast<uint32_t>(st.list_len_sync());
        }
        if (cnt_prev > shrink_at) {
          csync();
          shrink_row();
          cnt_prev = S.v->cnt;
        }
      } else if (!c.stream) {
        fold(sacc0, sacc1, s);
        for (int vb = warp * 32; vb < nvec; vb += kThreads) {
          const int v = vb + lane;
          const bool valid = v < nvec;
          float x[EPV];
          if (valid) {
            Tr::unpack(sv[v], x);
          } else {
#pragma unroll
            for (int i = 0; i < EPV; ++i) x[i] = -kInf;
          }
          st.template process<EPV>(c, x, tbase + v * EPV, valid, m, s, thr_y, thr_key);
        }
      } else {
        // per-beam top-K rows (and vocab-sharded partial rows) keep every element
        fold(sacc0, sacc1, s);
        for (int sb = 0; sb < nvec; sb += P.sub_vecs) {
          const int send = min(nvec, sb + P.sub_vecs);
          for (int vb = sb + warp * 32; vb < send; vb += kThreads) {
            const int v = vb + lane;
            const bool valid = v < send;
            float x[EPV];
            if (valid) {
              Tr::unpack(sv[v], x);
            } else {
#pragma unroll
              for (int i = 0; i < EPV; ++i) x[i] = -kInf;
            }
            st.template process<EPV>(c, x, tbase + v * EPV, valid, m, s, thr_y, thr_key);
          }
          if (st.list_len_sync() > kKeyCap - P.sub_vecs * EPV) shrink_row();
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&S.empty[cstage]);
      if (++cstage == P.stages) {
        cstage = 0;
        cphase ^= 1u;
      }
      ++consumed;
    }

    fold(sacc0, sacc1, s);
    GR_PROF_ADD(0, t_stream);
    GR_PROF_T(t_red);

    // ------------------------------------------------------------ row end
    if (c.excl) {
      // penalised tokens were left out of the stream; add their exact values
      const int nt = static_cast<int>(S.v->ntab);
      for (int jb = warp * 32; jb < nt; jb += kThreads) {
        const int j = jb + lane;
        const bool valid = j < nt;
        float y[1];
        y[0] = valid ? S.tab_y[j] : -kInf;
        if (valid) st.template lse_update<1>(y, m, s);
        if (c.stream) {
          bool pred = false;
          uint64_t key = 0;
          if (valid) {
            key = make_key(y[0], static_cast<uint32_t>(c.b) * static_cast<uint32_t>(P.V) +
                                     static_cast<uint32_t>(tok_of(P, S.tab_tok[j])));
            pred = key >= thr_key;
          }
          warp_append(pred, key, S.keys, &S.v->cnt, kKeyCap, &S.v->overflow);
        }
      }
    }
    // consumer-wide reduction of (m, s)
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float m2 = __shfl_xor_sync(0xFFFFFFFFu, m, o);
      const float s2 = __shfl_xor_sync(0xFFFFFFFFu, s, o);
      const float M = fmaxf(m, m2);
      if (M == -kInf) {
        s = 0.0f;
      } else {
        s = s * fast_exp2((m - M) * kLog2e) + s2 * fast_exp2((m2 - M) * kLog2e);
      }
      m = M;
    }
    if (lane == 0) {
      S.red_m[warp] = m;
      S.red_s[warp] = s;
    }
    if (tid == 0) {
      S.v->abort_snap = S.v->abort;
      if (!P.partial_only) {
        S.v->tau_pref = tau_pref;
        if (c.constrained) S.v->thr_key = tau_pref;      // candidates start from the request bound
      }
    }
    csync();
    // every thread combines the warp partials (same order, same result everywhere)
    float lse;
    {
      float M = -kInf;
#pragma unroll
      for (int w = 0; w < kWarps; ++w) M = fmaxf(M, S.red_m[w]);
      float tot = 0.0f;
      if (M > -kInf) {
#pragma unroll
        for (int w = 0; w < kWarps; ++w) tot += S.red_s[w] * fast_exp2((S.red_m[w] - M) * kLog2e);
      }
      lse = M + logf(tot);
      if (P.lse_in) lse = P.lse_in[c.row];   // vocab-sharded phase 2: the global normaliser
      if (tid == 0) {
        if (P.lse_out) P.lse_out[c.row] = lse;
        if (P.partial_only) P.partials[c.row] = make_float2(M, tot);
      }
    }
    GR_PROF_ADD(2, t_red);
    if (S.v->abort_snap) goto drain;
    GR_PROF_T(t_cand);

    if (!P.partial_only) {
      if (c.constrained) {
        st.constrained_candidates(c, lse);
      } else if (c.stream && P.K == 0) {
        st.unconstrained_candidates(c, lse);
      } else if (c.stream) {
        st.literal_candidates(c, lse);
      }
      GR_PROF_ADD(3, t_cand);
      GR_PROF_T(t_emit);
      if (tid == 0 && S.v->overflow) atomicOr(P.err, GR_DEVERR_OVERFLOW);
      if (c.stream) {
        // the row-local threshold was over value keys; only the request bound applies now
        if (tid == 0) S.v->thr_key = 0ull;
        csync();
      }
      // constrained rows were filtered against the request bound while they were scored
      st.emit(c, /*refilter=*/!c.constrained);
      GR_PROF_ADD(4, t_emit);
    }
    if (c.pen_active) {
      const int nt = static_cast<int>(S.v->ntab);
      for (int j = tid; j < nt; j += kThreads) S.bitmap[S.tab_tok[j] >> 5] = 0u;
    }
    csync();
  }
  GR_PROF_ADD(11, t_kernel);
  GR_PROF_FLUSH();
  return;

drain:
  // A bounded wait ran out: wait (bounded) for the producer to stop and for
  // the copies it issued that were not consumed, so that none lands after the
  // CTA has exited.
  if (tid == 0) {
    const uint64_t t0 = global_timer_ns();
    while (!*reinterpret_cast<volatile int*>(&S.v->producer_done) && global_timer_ns() - t0 < kWaitLimitNs) {
    }
    const long long issued = *reinterpret_cast<volatile long long*>(&S.v->issued);
    for (long long q = consumed; q < issued; ++q) {
      mbar_wait_bounded(&S.full[cstage], cphase);
      if (++cstage == P.stages) {
        cstage = 0;
        cphase ^= 1u;
      }
    }
  }
  csync();
}

#include "gr_step_ws.cuh"
#include "gr_step_select_ws.cuh"

// ---------------------------------------------------------------- merge kernel
// One CTA of kThreads threads per request: gathers the request's per-row
// candidate slots, keeps the canonical top-2B (radix select over the keys),
// sorts them and writes candidates, new beams with their child trie nodes and
// the forked token table (serving_engine.py:566-590, llm.py:256-276).
constexpr int kMergeMaxBeams = 4096;
constexpr int kMergeCap = 16384;         // request candidates gathered into shared memory at once
constexpr int kMergeTop = kKeyCap / 2;   // the kept keys (k2 <= kKeyCap / 2)

struct MergeSmem {
  uint64_t* keys;      // [kMergeCap] gathered keys
  uint64_t* top;       // [kMergeTop] the kept top-2B
  int* dec_tok;        // [kMergeTop] token of sorted candidate i
  int* dec_par;        // [kMergeTop] parent beam of sorted candidate i
  uint32_t* prefix;    // [NB + 1] exclusive prefix of the rows' counts
  uint32_t* rc;        // [NB] the rows' counts
  uint16_t* row_of;    // [kMergeCap] row of gathered index i
  SelectScratch* sel;
  uint32_t* wsum;      // [kWarps]
  uint32_t* cnt;       // [4] gathered, kept, real total
};

__host__ __device__ inline size_t merge_smem_bytes(int NB) {
  return align128(size_t(kMergeCap) * 8) + align128(size_t(kMergeTop) * 8) + 2 * align128(size_t(kMergeTop) * 4) +
         align128(size_t(NB + 1) * 4) + align128(size_t(NB) * 4) + align128(size_t(kMergeCap) * 2) +
         align128(sizeof(SelectScratch)) + align128(kWarps * 4) + 128;
}

__device__ __forceinline__ int row_of_index(const uint32_t* prefix, int NB, uint32_t i) {
  int lo = 0, hi = NB;                 // prefix[lo] <= i < prefix[hi]
  while (hi - lo > 1) {
    const int mid = (lo + hi) >> 1;
    if (prefix[mid] <= i) lo = mid; else hi = mid;
  }
  return lo;
}

// Trie child of (parent node, token) by a binary search of the CSR children
// (rows whose keys carry the token: per-beam top-K steps).
__device__ __forceinline__ int child_by_search(const Params& P, const int* rec, int tok) {
  const int pn = rec[kMNode];
  if (pn == GR_NODE_UNCONSTRAINED) return GR_NODE_UNCONSTRAINED;
  if (pn < 0) return GR_NODE_DEAD;
  int lo = rec[kMC0], hi = rec[kMC1];
  const int c1 = hi;
  while (lo < hi) {
    const int mid = (lo + hi) >> 1;
    if (__ldg(P.child_tok + mid) < tok) lo = mid + 1; else hi = mid;
  }
  return (lo < c1 && __ldg(P.child_tok + lo) == tok) ? __ldg(P.child_node + lo) : GR_NODE_DEAD;
}

__global__ void __launch_bounds__(kThreads) merge_kernel(const __grid_constant__ Params P) {
  unsigned char* smem_raw = g_smem;
  MergeSmem M;
  {
    size_t o = 0;
    M.keys = reinterpret_cast<uint64_t*>(smem_raw + o); o += align128(size_t(kMergeCap) * 8);
    M.top = reinterpret_cast<uint64_t*>(smem_raw + o); o += align128(size_t(kMergeTop) * 8);
    M.dec_tok = reinterpret_cast<int*>(smem_raw + o); o += align128(size_t(kMergeTop) * 4);
    M.dec_par = reinterpret_cast<int*>(smem_raw + o); o += align128(size_t(kMergeTop) * 4);
    const int rows = max(P.NB, P.slot_rows);
    M.prefix = reinterpret_cast<uint32_t*>(smem_raw + o); o += align128(size_t(rows + 1) * 4);
    M.rc = reinterpret_cast<uint32_t*>(smem_raw + o); o += align128(size_t(rows) * 4);
    M.row_of = reinterpret_cast<uint16_t*>(smem_raw + o); o += align128(size_t(kMergeCap) * 2);
    M.sel = reinterpret_cast<SelectScratch*>(smem_raw + o); o += align128(sizeof(SelectScratch));
    M.wsum = reinterpret_cast<uint32_t*>(smem_raw + o); o += align128(kWarps * 4);
    M.cnt = reinterpret_cast<uint32_t*>(smem_raw + o);
  }
  const int r = blockIdx.x, tid = threadIdx.x, lane = lane_id(), warp = warp_id();
  const int NB = P.NB, k2 = P.k2;
  const int S = P.slot_rows;   // slots gathered per request (rows, or shards)
  pdl_wait();   // the step kernel's row slots, counts and bounds
  pdl_trigger();   // the next step's row records may launch (they wait for this grid)
  if (P.clear_err) {
    // GR_STEP_CLEAR_ERR: the bad node ids row_meta_kernel found in this
    // request's rows (its records are complete: the step kernel waited for it)
    for (int b = tid; b < NB; b += blockDim.x)
      if (P.meta[(static_cast<size_t>(r) * NB + b) * kMetaWords + kMBad]) atomicOr(P.err, GR_DEVERR_BAD_NODE);
  }
#ifdef GR_PHASE_PROFILE
  long long mt[8];
  int mq = 0;
#define GR_MPROF() do { if (tid == 0 && mq < 8) mt[mq++] = clock64(); } while (0)
#else
#define GR_MPROF() do { } while (0)
#endif
  GR_MPROF();
  // ---- per-slot counts (no count array: every slot full, zero keys empty) and their exclusive prefix
  const int per = (S + kThreads - 1) / kThreads;
  const int b0 = min(tid * per, S), b1 = min(b0 + per, S);
  uint32_t local = 0;
  for (int b = b0; b < b1; ++b) {
    const uint32_t c = P.rowcnt ? min(__ldcg(P.rowcnt + static_cast<size_t>(r) * NB + b), static_cast<unsigned>(P.slot_cap))
                                : static_cast<uint32_t>(P.slot_cap);
    M.rc[b] = c;
    local += c;
  }
  uint32_t inc = local;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const uint32_t v = __shfl_up_sync(0xFFFFFFFFu, inc, o);
    if (lane >= o) inc += v;
  }
  if (lane == 31) M.wsum[warp] = inc;
  if (tid == 0) {
    M.cnt[0] = 0;
    M.cnt[1] = 0;
    M.cnt[2] = 0;
  }
  csync();
  if (tid == 0) {
    uint32_t acc = 0;
    for (int w = 0; w < kWarps; ++w) {
      const uint32_t t = M.wsum[w];
      M.wsum[w] = acc;
      acc += t;
    }
    M.prefix[S] = acc;
  }
  csync();
  uint32_t base = M.wsum[warp] + inc - local;
  for (int b = b0; b < b1; ++b) {
    M.prefix[b] = base;
    base += M.rc[b];
  }
  csync();
  const int n_all = static_cast<int>(M.prefix[S]);
  int k = min(k2, n_all);
  // the request's final bound: at least 2B gathered keys are >= it (it is the
  // 2B-th key of some row's own list), so smaller keys take no part
  const uint64_t tau = __ldcg(P.tau + r);
  // slot b of this request starts at slots + b * slot_step
  const unsigned long long* slots = P.buf + static_cast<size_t>(r) * P.slot_sr * static_cast<size_t>(k2);
  const size_t slot_step = static_cast<size_t>(P.slot_sb) * static_cast<size_t>(k2);
  const uint32_t* prefix = M.prefix;
  const uint32_t* rc = M.rc;
  int dummy = 0;
  GR_MPROF();
  // ---- canonical top-2B
  int n = 0;   // keys >= tau gathered into shared memory
  // the shared-memory path takes every flat list (its keys >= tau almost always
  // fit) and every slot grid whose keys all fit; an overflow falls back below
  bool smem_path = (S == 1) || (n_all <= kMergeCap);
  if (smem_path) {
    // row of every gathered index (one warp per row), then a flat gather with
    // kU independent loads per thread in flight
    if (S > 1) {
      for (int b = warp; b < S; b += kWarps)
        for (uint32_t j = lane; j < rc[b]; j += 32) M.row_of[prefix[b] + j] = static_cast<uint16_t>(b);
      csync();
    }
    constexpr int kU = 16;
    for (int base0 = 0; base0 < n_all; base0 += kThreads * kU) {
      // addresses first, then every load, then the uses: no load waits for another
      const unsigned long long* src[kU];
#pragma unroll
      for (int u = 0; u < kU; ++u) {
        const int i = min(base0 + u * kThreads + tid, n_all - 1);
        const int b = (S > 1) ? M.row_of[i] : 0;
        src[u] = slots + static_cast<size_t>(b) * slot_step + (static_cast<uint32_t>(i) - prefix[b]);
      }
      uint64_t kv[kU];
#pragma unroll
      for (int u = 0; u < kU; ++u) kv[u] = __ldcg(src[u]);
      uint32_t mask = 0;
#pragma unroll
      for (int u = 0; u < kU; ++u)
        if (base0 + u * kThreads + tid < n_all && kv[u] >= tau && kv[u] != 0ull) mask |= 1u << u;
      warp_append_n<kU>(mask, kv, M.keys, &M.cnt[0], kMergeCap, reinterpret_cast<int*>(&M.cnt[2]));
    }
    csync();
    smem_path = M.cnt[2] == 0;   // no key was dropped
  }
  if (smem_path) {
    n = static_cast<int>(M.cnt[0]);
    k = min(k, n);
    GR_MPROF();
    uint64_t* keys = M.keys;
    Cut cut{0ull, 0};   // keeps every key
    if (n > k) cut = cta_radix_select([keys](int i) { return keys[i]; }, n, k, M.sel);
    GR_MPROF();
    constexpr int kC = 16;
    for (int base0 = 0; base0 < n; base0 += kThreads * kC) {
      uint64_t kv[kC];
      uint32_t mask = 0;
#pragma unroll
      for (int u = 0; u < kC; ++u) {
        const int i = base0 + u * kThreads + tid;
        kv[u] = (i < n) ? keys[i] : 0ull;
        if (i < n && cut.keep(kv[u])) mask |= 1u << u;
      }
      warp_append_n<kC>(mask, kv, M.top, &M.cnt[1], kMergeTop, &dummy);
    }
    csync();
  } else {
    auto keyf = [slots, prefix, S, slot_step](int i) -> uint64_t {
      const int b = row_of_index(prefix, S, static_cast<uint32_t>(i));
      return __ldcg(slots + static_cast<size_t>(b) * slot_step + (static_cast<uint32_t>(i) - prefix[b]));
    };
    GR_MPROF();
    Cut cut{0ull, 0};
    if (n_all > k) cut = cta_radix_select(keyf, n_all, k, M.sel);
    GR_MPROF();
    for (int ib = warp * 32; ib < n_all; ib += kThreads) {
      const int i = ib + lane;
      const uint64_t key = (i < n_all) ? keyf(i) : 0ull;
      warp_append(i < n_all && key != 0ull && cut.keep(key), key, M.top, &M.cnt[1], kMergeTop, &dummy);
    }
    csync();
    k = min(k, static_cast<int>(M.cnt[1]));
  }
  GR_MPROF();
  // ---- descending order: rank sort for small k, bitonic otherwise
  if (k <= kThreads) {
    const uint64_t mine = (tid < k) ? M.top[tid] : 0ull;
    int rank = 0;
    int j = 0;
    for (; j + 8 <= k; j += 8) {
#pragma unroll
      for (int u = 0; u < 8; ++u) rank += (M.top[j + u] > mine);
    }
    for (; j < k; ++j) rank += (M.top[j] > mine);
    if (tid < k) M.keys[rank] = mine;
    csync();
  } else {
    int P2 = 1;
    while (P2 < k) P2 <<= 1;
    for (int i = tid; i < P2; i += kThreads) M.keys[i] = (i < k) ? M.top[i] : 0ull;
    csync();
    if (P2 == 2 * kThreads) cta_bitonic_sort_regs_desc<2>(M.keys);
    else if (P2 == 4 * kThreads) cta_bitonic_sort_regs_desc<4>(M.keys);
    else if (P2 == 8 * kThreads) cta_bitonic_sort_regs_desc<8>(M.keys);
    else cta_bitonic_sort_desc(M.keys, P2);
  }
  GR_MPROF();
  if (P.keys_out) {
    // vocab-sharded phase 2: this shard's top-2B keys in canonical order (key
    // descending), zero padded: the same bytes whichever step kernel ran
    for (int i = tid; i < k2; i += kThreads) P.keys_out[static_cast<size_t>(r) * k2 + i] = (i < k) ? M.keys[i] : 0ull;
    return;
  }
  // ---- outputs: kO candidates per thread at a time, every load of a batch
  // issued before any of them is used
  const int B = P.B, T = P.T;
  constexpr int kO = 8;
  for (int i0 = tid; i0 < k2; i0 += kThreads * kO) {
    int par[kO], x[kO], pn[kO], c0[kO];
    float sc[kO];
#pragma unroll
    for (int u = 0; u < kO; ++u) {
      const int i = i0 + u * kThreads;
      sc[u] = -kInf;
      par[u] = -1;
      x[u] = 0;
      if (i < k) {
        const uint64_t key = M.keys[i];
        const uint32_t flat = key_flat(key);
        sc[u] = key_score(key);
        par[u] = static_cast<int>(flat / static_cast<uint32_t>(P.V));
        x[u] = static_cast<int>(flat - static_cast<uint32_t>(par[u]) * static_cast<uint32_t>(P.V));
      }
    }
#pragma unroll
    for (int u = 0; u < kO; ++u) {
      const int* rec = P.meta + static_cast<size_t>(r * NB + max(par[u], 0)) * kMetaWords;
      pn[u] = __ldcg(rec + kMNode);
      c0[u] = __ldcg(rec + kMC0);
    }
    int tok[kO], child[kO];
#pragma unroll
    for (int u = 0; u < kO; ++u) {
      const int i = i0 + u * kThreads;
      tok[u] = -1;
      child[u] = GR_NODE_DEAD;
      if (par[u] >= 0 && P.K == 0 && pn[u] >= 0) {
        // catalog row: the key carries the child's CSR position
        tok[u] = __ldg(P.child_tok + c0[u] + x[u]);
        if (i < B) child[u] = __ldg(P.child_node + c0[u] + x[u]);
      }
    }
#pragma unroll
    for (int u = 0; u < kO; ++u) {
      const int i = i0 + u * kThreads;
      if (i >= k2) continue;
      if (par[u] >= 0 && !(P.K == 0 && pn[u] >= 0)) {
        tok[u] = x[u];
        if (i < B)
          child[u] = (pn[u] == GR_NODE_UNCONSTRAINED)
                         ? GR_NODE_UNCONSTRAINED
                         : child_by_search(P, P.meta + static_cast<size_t>(r * NB + par[u]) * kMetaWords, tok[u]);
      }
      if (i < kMergeTop) {
        M.dec_tok[i] = tok[u];
        M.dec_par[i] = par[u];
      }
      P.cand_score[static_cast<size_t>(r) * k2 + i] = sc[u];
      P.cand_token[static_cast<size_t>(r) * k2 + i] = tok[u];
      P.cand_parent[static_cast<size_t>(r) * k2 + i] = par[u];
      if (i < B) {
        P.sel_score[static_cast<size_t>(r) * B + i] = sc[u];
        P.sel_token[static_cast<size_t>(r) * B + i] = tok[u];
        P.sel_parent[static_cast<size_t>(r) * B + i] = par[u];
        P.sel_node[static_cast<size_t>(r) * B + i] = child[u];
      }
    }
  }
  if (P.hist_out) {
    csync();
    const int W = T + 1;
    constexpr int kH = 8;   // entries per thread per batch, loads first
    for (int idx0 = tid; idx0 < B * W; idx0 += kThreads * kH) {
      int v[kH];
#pragma unroll
      for (int u = 0; u < kH; ++u) {
        const int idx = idx0 + u * kThreads;
        const int i = idx / W, t = idx - i * W;
        v[u] = -1;
        if (idx < B * W && i < k) {
          const int par = M.dec_par[i];
          v[u] = (t < T) ? __ldg(P.hist + (static_cast<size_t>(r) * NB + par) * T + t) : M.dec_tok[i];
        }
      }
#pragma unroll
      for (int u = 0; u < kH; ++u) {
        const int idx = idx0 + u * kThreads;
        if (idx < B * W) P.hist_out[static_cast<size_t>(r) * B * W + idx] = v[u];
      }
    }
  }
#ifdef GR_PHASE_PROFILE
  GR_MPROF();
  if (tid == 0 && r < 512)   // merge counters sit after the step kernels' CTAs
    for (int q = 1; q < mq; ++q) g_phase[512 + r][q] += static_cast<unsigned long long>(mt[q] - mt[q - 1]);
#endif
}

// ============================================================== host side
struct DeviceInfo {
  int sms = 0;
  int smem_optin = 0;
  int smem_per_sm = 0;
  int smem_reserved = 0;
  int major = 0;
  bool attr_set[3] = {false, false, false};
  bool ws_attr_set[3] = {false, false, false};
  bool sel_attr_set[3] = {false, false, false};
  bool merge_attr_set = false;
};

static DeviceInfo g_dev[64];
// Guards the per-device records (filled on a device's first call) and their
// kernel-attribute flags: calls may come from several host threads.
static std::mutex g_dev_mu;

static int device_info(DeviceInfo** out) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return GR_ERR_NO_DEVICE;
  if (dev < 0 || dev >= 64) return GR_ERR_NO_DEVICE;
  std::lock_guard<std::mutex> lock(g_dev_mu);
  DeviceInfo& d = g_dev[dev];
  if (d.sms == 0) {
    int sms = 0, smem = 0, major = 0;
    if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) return GR_ERR_CUDA;
    if (cudaDeviceGetAttribute(&smem, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev) != cudaSuccess) return GR_ERR_CUDA;
    if (cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev) != cudaSuccess) return GR_ERR_CUDA;
    int per_sm = 0, reserved = 0;
    if (cudaDeviceGetAttribute(&per_sm, cudaDevAttrMaxSharedMemoryPerMultiprocessor, dev) != cudaSuccess)
      return GR_ERR_CUDA;
    if (cudaDeviceGetAttribute(&reserved, cudaDevAttrReservedSharedMemoryPerBlock, dev) != cudaSuccess)
      return GR_ERR_CUDA;
    d.smem_per_sm = per_sm;
    d.smem_reserved = reserved;
    d.smem_optin = smem;
    d.major = major;
    d.sms = sms;
  }
  if (d.major != 10) return GR_ERR_NO_DEVICE;
  *out = &d;
  return GR_OK;
}

// Workspace: tau [R] u64 | row counts [R*NB] u32 | row metadata [R*NB][kMetaWords] i32 |
// row slots [R*NB][2B] u64.
static size_t ws_tau_bytes(int R) { return align128(size_t(R) * 8 + 8); }   // + the row counter
static size_t ws_cnt_bytes(int R, int NB) { return align128(size_t(R) * NB * 4); }
static size_t ws_meta_bytes(int R, int NB) { return align128(size_t(R) * NB * kMetaWords * 4); }
// Penalty tables of the selecting kernel: steps with processed log-probs, a
// history of at most sel::kPenCap tokens and no per-beam top-K.
static int ws_tab_words(const gr_step_desc* d) {
  const bool used = d->logprobs_mode == GR_LOGPROBS_PROCESSED && d->hist_len >= 1 &&
                    d->hist_len <= sel::kPenCap && d->per_beam_k == 0;
  return used ? (d->hist_len + 31) / 32 * 32 : 0;
}
static size_t ws_tab_bytes(const gr_step_desc* d) {
  return align128(size_t(d->num_requests) * d->num_beams * 2 * size_t(ws_tab_words(d)) * 4);
}

static int validate(const gr_step_desc* d) {
  if (!d) return GR_ERR_NULL;
  if (d->num_requests < 1 || d->num_beams < 1 || d->beam_width < 1) return GR_ERR_BAD_DESC;
  if (d->vocab_size < 1 || d->vocab_local < 1 || d->vocab_offset < 0 || d->vocab_stride < 0) return GR_ERR_BAD_DESC;
  if (d->flags & ~GR_STEP_CLEAR_ERR) return GR_ERR_BAD_DESC;
  // the last local column's token: vocab_offset + (vocab_local - 1) * stride < vocab_size
  const long long vstride = d->vocab_stride > 1 ? d->vocab_stride : 1;
  if (static_cast<long long>(d->vocab_offset) + (d->vocab_local - 1) * vstride >= d->vocab_size) return GR_ERR_BAD_DESC;
  if (d->row_stride < d->vocab_local) return GR_ERR_BAD_DESC;
  if (d->logit_dtype < GR_DTYPE_F32 || d->logit_dtype > GR_DTYPE_F16) return GR_ERR_DTYPE;
  if (d->logprobs_mode != GR_LOGPROBS_RAW && d->logprobs_mode != GR_LOGPROBS_PROCESSED) return GR_ERR_DTYPE;
  if (d->per_beam_k < 0 || d->per_beam_k > d->vocab_local) return GR_ERR_BAD_DESC;
  if (d->hist_len < 0 || d->num_nodes < 0 || d->num_edges < 0) return GR_ERR_BAD_DESC;
  if (d->eos_token_id < -1 || d->eos_token_id >= d->vocab_size) return GR_ERR_BAD_DESC;
  // flat index parent*V + token must fit in 32 bits
  if (static_cast<unsigned long long>(d->num_beams) * static_cast<unsigned long long>(d->vocab_size) >
      0xFFFFFFFFull)
    return GR_ERR_UNSUPPORTED;
  // shared-memory key list: 2B (+ streamed slack) must fit beside one batch
  const int k2 = 2 * d->beam_width;
  if (k2 > kKeyCap / 2) return GR_ERR_UNSUPPORTED;
  const int kk = (k2 > d->per_beam_k ? k2 : d->per_beam_k) + kSlack;
  if (kk + 32 * 8 > kKeyCap) return GR_ERR_UNSUPPORTED;   // room for one warp-wide batch of 2-byte logits
  if (d->num_edges > 0x7FFFFFFFll) return GR_ERR_UNSUPPORTED;
  if (d->num_beams > kMergeMaxBeams) return GR_ERR_UNSUPPORTED;
  return GR_OK;
}

// Test hook (GR_TEST_STALL_COPIES=1): the step kernels' producers issue no
// bulk copies, so the consumers' bounded waits run out and the call reports
// GR_DEVERR_TIMEOUT instead of its result.  Tests use it to check the
// expiry path; nothing else sets it.
static int stall_copies_requested() {
  const char* e = std::getenv("GR_TEST_STALL_COPIES");
  return (e != nullptr && e[0] == '1') ? 1 : 0;
}

static void fill_params(Params& P, const gr_step_desc* d, const gr_step_io* io) {
  P.R = d->num_requests;
  P.NB = d->num_beams;
  P.B = d->beam_width;
  P.V = d->vocab_size;
  P.VL = d->vocab_local;
  P.voff = d->vocab_offset;
  P.vstride = d->vocab_stride > 1 ? d->vocab_stride : 1;
  P.row_stride = d->row_stride;
  P.mode = d->logprobs_mode;
  P.K = d->per_beam_k;
  P.eos = d->eos_token_id;
  P.T = d->hist_len;
  P.N = d->num_nodes;
  P.logits = io->logits;
  P.cum = io->cum;
  P.node = io->node;
  P.row_ptr = reinterpret_cast<const long long*>(io->row_ptr);
  P.child_tok = io->child_tok;
  P.child_node = io->child_node;
  P.temp = io->temperature;
  P.rep = io->rep_penalty;
  P.pres = io->pres_penalty;
  P.freq = io->freq_penalty;
  P.hist = io->hist_in;
  P.cand_score = io->cand_score;
  P.cand_token = io->cand_token;
  P.cand_parent = io->cand_parent;
  P.sel_score = io->sel_score;
  P.sel_token = io->sel_token;
  P.sel_parent = io->sel_parent;
  P.sel_node = io->sel_node;
  P.eos_score = io->eos_score;
  P.hist_out = io->hist_out;
  P.lse_out = io->lse;
  P.err = io->err;
  P.k2 = 2 * d->beam_width;
  P.kk = (P.k2 > P.K ? P.k2 : P.K) + kSlack;
  {
    // streamed rows add at most sub_vecs * EPV keys between shrinks back to kk
    const int epv = (d->logit_dtype == GR_DTYPE_F32) ? 4 : 8;
    const int room = (kKeyCap - P.kk < kBatch) ? kKeyCap - P.kk : kBatch;
    P.sub_vecs = (room / epv) / 32 * 32;
    if (P.sub_vecs < 32) P.sub_vecs = 32;
  }
  P.pen = (io->rep_penalty || io->pres_penalty || io->freq_penalty) ? 1 : 0;
  P.bm_words = (d->vocab_local + 31) / 32 + 1;
  P.tab_cap = P.pen ? ((d->hist_len > 0 ? d->hist_len : 1) + 31) / 32 * 32 : 0;
  P.win_bytes = (d->num_nodes > 0 && P.K == 0) ? kWinBytes : 0;
  P.partial_only = 0;
  P.stall_copies = stall_copies_requested();
  P.clear_err = (d->flags & GR_STEP_CLEAR_ERR) ? 1 : 0;
  P.partials = nullptr;
  P.lse_in = nullptr;
  P.keys_out = nullptr;
  P.slot_rows = 1;
  P.slot_sr = d->num_beams;
  P.slot_sb = 1;
  P.slot_cap = d->num_beams * 2 * d->beam_width;
}

// Two CTAs per SM when at least three ring stages fit beside the fixed
// shared-memory pieces (one CTA's row-end work then overlaps the other CTA's
// streaming); otherwise one CTA per SM with as many stages as fit.
static int pick_stages(const Params& P, const DeviceInfo* dev, int* ctas_per_sm) {
  const size_t optin = static_cast<size_t>(dev->smem_optin);
  const size_t per_sm = static_cast<size_t>(dev->smem_per_sm);
  const size_t rsv = static_cast<size_t>(dev->smem_reserved);
  for (int st = kMaxStages; st >= 3; --st) {
    const size_t b = smem_bytes(st, P.win_bytes, P.bm_words, P.tab_cap, P.pen);
    if (b <= optin && 2 * (b + rsv) <= per_sm) {
      *ctas_per_sm = 2;
      return st;
    }
  }
  for (int st = kMaxStages; st >= 2; --st) {
    if (smem_bytes(st, P.win_bytes, P.bm_words, P.tab_cap, P.pen) <= optin) {
      *ctas_per_sm = 1;
      return st;
    }
  }
  return 0;
}

template <typename TL>
static int launch_fused(Params& P, DeviceInfo* dev, int dtype_idx, cudaStream_t stream) {
  int per = 1;
  const int stages = pick_stages(P, dev, &per);
  if (stages == 0) return GR_ERR_UNSUPPORTED;
  P.stages = stages;
  const size_t smem = smem_bytes(stages, P.win_bytes, P.bm_words, P.tab_cap, P.pen);
  std::unique_lock<std::mutex> attr_lock(g_dev_mu);
  if (!dev->attr_set[dtype_idx]) {
    if (cudaFuncSetAttribute(fused_step_kernel<TL>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             dev->smem_optin) != cudaSuccess)
      return GR_ERR_CUDA;
    dev->attr_set[dtype_idx] = true;
  }
  attr_lock.unlock();
  int occ = 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, fused_step_kernel<TL>, kBlock, smem) != cudaSuccess)
    return GR_ERR_CUDA;
  if (occ < 1) return GR_ERR_UNSUPPORTED;
  if (occ < per) per = occ;
  const int total = P.R * P.NB;
  const int slots = dev->sms * per;
  const int grid = total < slots ? total : slots;
  if (launch_pdl(fused_step_kernel<TL>, dim3(grid), dim3(kBlock), smem, stream, P) != cudaSuccess) return GR_ERR_CUDA;
  return GR_OK;
}

// Launch with programmatic stream serialization (the kernel calls pdl_wait()
// before it reads what the previous kernel in the stream wrote).
template <typename... KArgs, typename... Args>
static cudaError_t launch_pdl(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t s,
                              Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kern, std::forward<Args>(args)...);
}

// The warp-specialised kernel takes steps whose rows need no streamed
// selection and no penalty exclusion; the selecting one steps without a
// catalog (every row streamed) within its table and list limits.
// GR_BEAM_KERNEL=stream|ws|select forces one kernel (ws and select only where
// eligible); anything else selects automatically.
static bool ws_eligible(const Params& P) {
  return P.K == 0 && !(P.mode == kModeProcessed && P.pen && P.T > 0);
}

static bool select_eligible(const Params& P, int es) {
  if (P.K != 0 || P.N != 0 || P.partial_only || P.lse_in != nullptr) return false;
  if (P.pen && P.T > 0 && P.mode == kModeProcessed && P.T > sel::kPenCap) return false;
  if (P.kk + kThreads * (es == 4 ? 4 : 8) > kKeyCap) return false;            // one selection round beside kk keys
  return static_cast<long long>(P.VL) * es <= static_cast<long long>(sel::kMaxRowStages) * sel::kStage;
}

static int kernel_choice() {
  const char* e = std::getenv("GR_BEAM_KERNEL");
  if (e == nullptr) return 0;
  if (std::strcmp(e, "stream") == 0) return 1;
  if (std::strcmp(e, "ws") == 0) return 2;
  if (std::strcmp(e, "select") == 0) return 3;
  return 0;
}

template <typename TL>
static int launch_fused_select(Params& P, DeviceInfo* dev, int dtype_idx, cudaStream_t stream) {
  int stages = 0;
  for (int st = kMaxStages; st >= 3; --st) {
    if (sel::smem_bytes(st) <= static_cast<size_t>(dev->smem_optin)) {
      stages = st;
      break;
    }
  }
  if (stages == 0) return launch_fused<TL>(P, dev, dtype_idx, stream);
  P.stages = stages;
  const size_t smem = sel::smem_bytes(stages);
  std::unique_lock<std::mutex> attr_lock(g_dev_mu);
  if (!dev->sel_attr_set[dtype_idx]) {
    if (cudaFuncSetAttribute(fused_select_ws_kernel<TL>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             dev->smem_optin) != cudaSuccess)
      return GR_ERR_CUDA;
    dev->sel_attr_set[dtype_idx] = true;
  }
  attr_lock.unlock();
  const int total = P.R * P.NB;
  // the rows' penalty tables first (one warp per row), when penalties apply
  if (!sel::pen_used(P)) P.pen_tab = nullptr;
  if (P.pen_tab != nullptr &&
      launch_pdl(pen_table_kernel<TL>, dim3((total + 7) / 8), dim3(256), 0, stream, P) != cudaSuccess)
    return GR_ERR_CUDA;
  const int grid = total < dev->sms ? total : dev->sms;
  if (launch_pdl(fused_select_ws_kernel<TL>, dim3(grid), dim3(sel::kBlockSel), smem, stream, P) != cudaSuccess)
    return GR_ERR_CUDA;
  return GR_OK;
}

template <typename TL>
static int launch_fused_ws(Params& P, DeviceInfo* dev, int dtype_idx, cudaStream_t stream) {
  int stages = 0;
  for (int st = ws::kMaxStagesWs; st >= 3; --st) {
    if (ws::smem_bytes(st) <= static_cast<size_t>(dev->smem_optin)) {
      stages = st;
      break;
    }
  }
  if (stages == 0) return launch_fused<TL>(P, dev, dtype_idx, stream);
  P.stages = stages;
  const size_t smem = ws::smem_bytes(stages);
  std::unique_lock<std::mutex> attr_lock(g_dev_mu);
  if (!dev->ws_attr_set[dtype_idx]) {
    if (cudaFuncSetAttribute(fused_step_ws_kernel<TL>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             dev->smem_optin) != cudaSuccess)
      return GR_ERR_CUDA;
    dev->ws_attr_set[dtype_idx] = true;
  }
  attr_lock.unlock();
  const int total = P.R * P.NB;
  const int grid = total < dev->sms ? total : dev->sms;
  if (launch_pdl(fused_step_ws_kernel<TL>, dim3(grid), dim3(ws::kBlockWs), smem, stream, P) != cudaSuccess)
    return GR_ERR_CUDA;
  return GR_OK;
}

template <typename TL>
static int launch_step_kernel(Params& P, DeviceInfo* dev, int dtype_idx, cudaStream_t stream) {
  const int choice = kernel_choice();
  // steps without a catalog: the selecting kernel (its streamers never wait
  // on the selection)
  if ((choice == 0 || choice == 3) && select_eligible(P, sizeof(TL)))
    return launch_fused_select<TL>(P, dev, dtype_idx, stream);
  // a given lse (vocab-sharded phase 2) leaves only row-end work: the streaming
  // kernel puts every consumer warp on it (GR_BEAM_KERNEL=ws keeps the other)
  const bool ws = ws_eligible(P) && (P.lse_in == nullptr ? choice != 1 : choice == 2);
  if (ws) return launch_fused_ws<TL>(P, dev, dtype_idx, stream);
  return launch_fused<TL>(P, dev, dtype_idx, stream);
}

static int launch_merge(const Params& P, DeviceInfo* dev, cudaStream_t stream) {
  const size_t smem = merge_smem_bytes(max(P.NB, P.slot_rows));
  if (smem > static_cast<size_t>(dev->smem_optin)) return GR_ERR_UNSUPPORTED;
  if (!dev->merge_attr_set) {
    if (cudaFuncSetAttribute(merge_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, dev->smem_optin) !=
        cudaSuccess)
      return GR_ERR_CUDA;
    dev->merge_attr_set = true;
  }
  if (launch_pdl(merge_kernel, dim3(P.R), dim3(kThreads), smem, stream, P) != cudaSuccess) return GR_ERR_CUDA;
  return GR_OK;
}

static int launch_by_dtype(Params& P, int dtype, DeviceInfo* dev, cudaStream_t stream) {
  switch (dtype) {
    case GR_DTYPE_F32: return launch_step_kernel<float>(P, dev, 0, stream);
    case GR_DTYPE_BF16: return launch_step_kernel<__nv_bfloat16>(P, dev, 1, stream);
    case GR_DTYPE_F16: return launch_step_kernel<__half>(P, dev, 2, stream);
    default: return GR_ERR_DTYPE;
  }
}

}  // namespace gr

namespace gr {
// Checks shared by the entry points, the workspace carve-up and the row
// metadata launch.  `need_out` / `need_logits`: the call writes the step's
// outputs / reads the logits.
static int setup_step(const gr_step_desc* d, const gr_step_io* io, void* workspace, size_t workspace_bytes,
                      cudaStream_t s, bool need_logits, bool need_out, Params& P, DeviceInfo** dev, float** lse_ws) {
  if (!d || !io) return GR_ERR_NULL;
  int v = validate(d);
  if (v != GR_OK) return v;
  if ((need_logits && !io->logits) || !io->cum || !io->node || !io->err) return GR_ERR_NULL;
  if (need_out && (!io->cand_score || !io->cand_token || !io->cand_parent)) return GR_ERR_NULL;
  if (need_out && (!io->sel_score || !io->sel_token || !io->sel_parent || !io->sel_node)) return GR_ERR_NULL;
  if (d->num_nodes > 0 && (!io->row_ptr || !io->child_tok || !io->child_node)) return GR_ERR_NULL;
  if (d->hist_len > 0 && !io->hist_in) return GR_ERR_NULL;
  const bool pen = io->rep_penalty || io->pres_penalty || io->freq_penalty;
  if (pen && d->hist_len > kPenTableMax) return GR_ERR_UNSUPPORTED;
  if (pen && (d->vocab_local + 31) / 32 + 1 > kMaxBitmapWords) return GR_ERR_UNSUPPORTED;
  if (!workspace) return GR_ERR_NULL;
  if (reinterpret_cast<uintptr_t>(workspace) & 255u) return GR_ERR_MISALIGNED;
  size_t need = 0;
  gr_beam_step_workspace_size(d, &need);
  if (workspace_bytes < need) return GR_ERR_WORKSPACE;
  v = device_info(dev);
  if (v != GR_OK) return v;
  fill_params(P, d, io);
  const int R = d->num_requests, NB = d->num_beams;
  unsigned char* ws = static_cast<unsigned char*>(workspace);
  size_t o = 0;
  P.tau = reinterpret_cast<unsigned long long*>(ws + o);
  P.row_counter = reinterpret_cast<unsigned int*>(P.tau + R);
  o += ws_tau_bytes(R);
  P.rowcnt = reinterpret_cast<unsigned int*>(ws + o); o += ws_cnt_bytes(R, NB);
  P.meta = reinterpret_cast<int*>(ws + o); o += ws_meta_bytes(R, NB);
  P.buf = reinterpret_cast<unsigned long long*>(ws + o); o += align128(size_t(R) * NB * size_t(P.k2) * 8);
  *lse_ws = reinterpret_cast<float*>(ws + o);
  o += align128(size_t(R) * NB * 4);
  P.req_hist = (P.k2 >= kReqHistMinK2) ? reinterpret_cast<unsigned int*>(ws + o) : nullptr;
  o += align128(size_t(R) * kReqHistBins * 4);
  P.tabw = ws_tab_words(d);
  P.pen_tab = (P.tabw > 0) ? reinterpret_cast<int*>(ws + o) : nullptr;
  const int rows = R * NB;
  if (launch_pdl(row_meta_kernel, dim3((rows + 255) / 256), dim3(256), 0, s, P) != cudaSuccess) return GR_ERR_CUDA;
  return GR_OK;
}

// Vocab-sharded: the rows' global log-sum-exp from every shard's (max, sumexp)
// partial, combined in shard order (the same value on every rank).
__global__ void __launch_bounds__(256) lse_combine_kernel(const float2* gathered, int shards, int rows, float* lse_ws,
                                                          float* lse_out) {
  const int row = blockIdx.x * blockDim.x + threadIdx.x;
  if (row >= rows) return;
  float M = -kInf;
  for (int k = 0; k < shards; ++k) M = fmaxf(M, gathered[static_cast<size_t>(k) * rows + row].x);
  float tot = 0.0f;
  if (M > -kInf)
    for (int k = 0; k < shards; ++k) {
      const float2 g = gathered[static_cast<size_t>(k) * rows + row];
      tot += g.y * fast_exp2((g.x - M) * kLog2e);
    }
  const float lse = M + logf(tot);
  lse_ws[row] = lse;
  if (lse_out) lse_out[row] = lse;
}
}  // namespace gr

using namespace gr;

extern "C" {

int32_t gr_abi_version(void) { return GR_ABI_VERSION; }

const char* gr_status_string(int32_t s) {
  switch (s) {
    case GR_OK: return "GR_OK";
    case GR_ERR_NULL: return "GR_ERR_NULL";
    case GR_ERR_BAD_DESC: return "GR_ERR_BAD_DESC";
    case GR_ERR_DTYPE: return "GR_ERR_DTYPE";
    case GR_ERR_MISALIGNED: return "GR_ERR_MISALIGNED";
    case GR_ERR_WORKSPACE: return "GR_ERR_WORKSPACE";
    case GR_ERR_UNSUPPORTED: return "GR_ERR_UNSUPPORTED";
    case GR_ERR_CUDA: return "GR_ERR_CUDA";
    case GR_ERR_NO_DEVICE: return "GR_ERR_NO_DEVICE";
    default: return "GR_ERR_UNKNOWN";
  }
}

int32_t gr_beam_step_workspace_size(const gr_step_desc* d, size_t* bytes) {
  if (!d || !bytes) return GR_ERR_NULL;
  const int v = validate(d);
  if (v != GR_OK) return v;
  const size_t slots = size_t(d->num_requests) * d->num_beams * size_t(2 * d->beam_width);
  *bytes = ws_tau_bytes(d->num_requests) + ws_cnt_bytes(d->num_requests, d->num_beams) +
           ws_meta_bytes(d->num_requests, d->num_beams) + align128(slots * 8) +
           align128(size_t(d->num_requests) * d->num_beams * 4) +
           align128(size_t(d->num_requests) * kReqHistBins * 4) + ws_tab_bytes(d);
  return GR_OK;
}


int32_t gr_beam_step(const gr_step_desc* d, const gr_step_io* io, void* workspace, size_t workspace_bytes,
                     void* stream) {
  gr::NvtxRange nvtx_range("gr_beam_step");
  Params P;
  DeviceInfo* dev = nullptr;
  float* lse_ws = nullptr;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  int v = setup_step(d, io, workspace, workspace_bytes, s, true, true, P, &dev, &lse_ws);
  if (v != GR_OK) return v;
  v = launch_by_dtype(P, d->logit_dtype, dev, s);
  if (v != GR_OK) return v;
  return launch_merge(P, dev, s);
}

#ifdef GR_PHASE_PROFILE
// Debug builds only: copy and clear the per-CTA phase counters.
int32_t gr_debug_phase_counters(void* host, size_t bytes) {
  if (bytes < sizeof(g_phase)) return GR_ERR_WORKSPACE;
  if (cudaMemcpyFromSymbol(host, g_phase, sizeof(g_phase)) != cudaSuccess) return GR_ERR_CUDA;
  static unsigned long long zeros[1024][kProfSlots];
  if (cudaMemcpyToSymbol(g_phase, zeros, sizeof(g_phase)) != cudaSuccess) return GR_ERR_CUDA;
  return GR_OK;
}
#endif

}  // extern "C"

// ------------------------------------------------------------------ no-alloc
// Scratch for gr_beam_step_noalloc: a fixed array in device memory that every
// GPU loading this library holds until the process exits.  Host code must not
// pass `g_noalloc_scratch` itself to a kernel (on the host it only names the
// symbol); the device address comes from cudaGetSymbolAddress, once per device.
namespace gr {
constexpr size_t kNoAllocScratchBytes = static_cast<size_t>(GR_NOALLOC_SCRATCH_BYTES);
static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];
static void* g_noalloc_ptr[64];
static std::mutex g_noalloc_mu;
}  // namespace gr

extern "C" {

int32_t gr_beam_step_noalloc(const gr_step_desc* d, const gr_step_io* io, void* stream) {
  gr::NvtxRange nvtx_range("gr_beam_step_noalloc");
  if (!d || !io) return GR_ERR_NULL;
  size_t need = 0;
  const int v = gr_beam_step_workspace_size(d, &need);
  if (v != GR_OK) return v;
  if (need > kNoAllocScratchBytes) return GR_ERR_WORKSPACE;    // beyond the built-in scratch
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return GR_ERR_NO_DEVICE;
  void* ptr = nullptr;
  {
    std::lock_guard<std::mutex> lock(g_noalloc_mu);
    ptr = g_noalloc_ptr[dev];
    if (ptr == nullptr) {
      // first call on this device (current device = dev): resolve the array's device address
      if (cudaGetSymbolAddress(&ptr, g_noalloc_scratch) != cudaSuccess || ptr == nullptr) return GR_ERR_CUDA;
      g_noalloc_ptr[dev] = ptr;
    }
  }
  // gr_beam_step clears the part of the scratch that must start at zero (the
  // per-request thresholds); every other byte it reads is written earlier in
  // the same call.
  return gr_beam_step(d, io, ptr, kNoAllocScratchBytes, stream);
}

int32_t gr_lse_partials(const gr_step_desc* d, const gr_step_io* io, float* partials, void* workspace,
                        size_t workspace_bytes, void* stream) {
  gr::NvtxRange nvtx_range("gr_lse_partials");
  if (!partials) return GR_ERR_NULL;
  if (d && d->flags != 0) return GR_ERR_BAD_DESC;   // flags are for the single-call step
  Params P;
  DeviceInfo* dev = nullptr;
  float* lse_ws = nullptr;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  int v = setup_step(d, io, workspace, workspace_bytes, s, true, false, P, &dev, &lse_ws);
  if (v != GR_OK) return v;
  P.partial_only = 1;
  P.partials = reinterpret_cast<float2*>(partials);
  P.lse_out = nullptr;
  P.eos_score = nullptr;
  return launch_by_dtype(P, d->logit_dtype, dev, s);
}

int32_t gr_shard_candidates(const gr_step_desc* d, const gr_step_io* io, const float* gathered_partials,
                            int32_t num_shards, uint64_t* shard_keys, void* workspace, size_t workspace_bytes,
                            void* stream) {
  gr::NvtxRange nvtx_range("gr_shard_candidates");
  if (!gathered_partials || !shard_keys) return GR_ERR_NULL;
  if (num_shards < 1) return GR_ERR_BAD_DESC;
  if (d && d->flags != 0) return GR_ERR_BAD_DESC;
  if (d && d->per_beam_k != 0) return GR_ERR_UNSUPPORTED;
  Params P;
  DeviceInfo* dev = nullptr;
  float* lse_ws = nullptr;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  int v = setup_step(d, io, workspace, workspace_bytes, s, true, false, P, &dev, &lse_ws);
  if (v != GR_OK) return v;
  const int rows = d->num_requests * d->num_beams;
  lse_combine_kernel<<<(rows + 255) / 256, 256, 0, s>>>(reinterpret_cast<const float2*>(gathered_partials),
                                                         num_shards, rows, lse_ws, io->lse);
  if (cudaGetLastError() != cudaSuccess) return GR_ERR_CUDA;
  P.lse_in = lse_ws;
  P.lse_out = nullptr;
  v = launch_by_dtype(P, d->logit_dtype, dev, s);
  if (v != GR_OK) return v;
  P.keys_out = reinterpret_cast<unsigned long long*>(shard_keys);
  return launch_merge(P, dev, s);
}

int32_t gr_merge_candidates(const gr_step_desc* d, const gr_step_io* io, const uint64_t* gathered_keys,
                            int32_t num_shards, void* workspace, size_t workspace_bytes, void* stream) {
  gr::NvtxRange nvtx_range("gr_merge_candidates");
  if (!gathered_keys) return GR_ERR_NULL;
  if (num_shards < 1 || num_shards > 65535) return GR_ERR_BAD_DESC;
  if (d && d->flags != 0) return GR_ERR_BAD_DESC;
  if (d && d->per_beam_k != 0) return GR_ERR_UNSUPPORTED;
  Params P;
  DeviceInfo* dev = nullptr;
  float* lse_ws = nullptr;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  int v = setup_step(d, io, workspace, workspace_bytes, s, false, true, P, &dev, &lse_ws);
  if (v != GR_OK) return v;
  // every shard's [R][2B] list is one slot of the request: slot k of request r
  // sits at gathered_keys + (k * R + r) * 2B
  P.buf = const_cast<unsigned long long*>(reinterpret_cast<const unsigned long long*>(gathered_keys));
  P.rowcnt = nullptr;
  P.slot_rows = num_shards;
  P.slot_sr = 1;
  P.slot_sb = d->num_requests;
  P.slot_cap = 2 * d->beam_width;
  return launch_merge(P, dev, s);
}

}  // extern "C"
