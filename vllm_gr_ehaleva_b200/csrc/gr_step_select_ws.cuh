// Warp-specialised step kernel for streamed rows: one CTA per SM, four warp
// roles, for steps without a catalog (every row's candidates are its own
// columns: unconstrained beams, with penalties and temperature or without).
//
//   warps 0..7    selectors  per ring stage: the candidate pass over the whole
//                            stage against a floor on the value (the request's
//                            running 2B-th key turned into a value through a
//                            lower bound of the row's lse that the streamers
//                            publish as they go), survivors kept in the row's
//                            key list (the Step helpers, named barrier 1 over
//                            these 256 threads)
//   next 16 warps streamers  (max, sum exp) of every row; after each stage every
//                            warp publishes the log-sum-exp of what it has seen,
//                            and the last one of the stage their combination
//   warp 24       producer   row scheduling, the row record, the row's penalty
//                            table (computed beforehand by pen_table_kernel)
//                            and flags, then the row body into the ring
//   warp 25       finisher   the row end of the rows the selectors hand over:
//                            the normaliser, the scores, the emission and the
//                            request histogram, while the selectors go on
//
// A ring stage is released once the 16 streaming and the 8 selecting warps
// are done with it, so the exponential sums never wait on the selection.
// Before its request has a bound a row keeps its own (the kk-th key of its
// list, barriers among the selectors) and the selectors end it themselves.
// A row that starts with the request's bound runs without barriers: per warp
// one reservation for the stage's few survivors in the row's slot; at its end
// the finisher takes it over, or, when its survivors did not fit the slot,
// the selectors select it exactly from global memory.  Penalised columns are
// left out of the stream (their processed values come from the table): the
// producer marks, per stage, the streaming threads whose vectors hold one.
// Included from gr_beam_step.cu.
#pragma once

// Optional per-role cycle counters (-DGR_PHASE_PROFILE, the debug build only).
#ifdef GR_PHASE_PROFILE
#define SEL_T(var) const long long var = clock64()
#define SEL_ADD(cond, slot, t0) \
  do { if (cond) atomicAdd(&S.v->prof[slot], static_cast<unsigned long long>(clock64() - (t0))); } while (0)
#define SEL_CNT(cond, slot, val) \
  do { if (cond) atomicAdd(&S.v->prof[slot], static_cast<unsigned long long>(val)); } while (0)
#else
#define SEL_T(var)
#define SEL_ADD(cond, slot, t0) do { } while (0)
#define SEL_CNT(cond, slot, val) do { } while (0)
#endif

namespace sel {
constexpr int kSelWarps = kWarps;                 // selectors are the Step helpers' kThreads
constexpr int kStrWarps = 16;
constexpr int kStrThreads = kStrWarps * 32;
constexpr int kProdWarp = kSelWarps + kStrWarps;
constexpr int kFinWarp = kProdWarp + 1;
constexpr int kBlockSel = (kFinWarp + 1) * 32;
constexpr int kVecPerThread = 4;                  // streamer vectors per stage
constexpr int kStage = kStrThreads * kVecPerThread * 16;   // 32 KB
constexpr int kStageVecs = kStage / 16;
constexpr int kSelVecs = kStageVecs / kThreads;   // selector vectors per stage (8)
constexpr int kSlots = 3;
constexpr int kPenCap = 128;                      // penalised columns per row
constexpr int kTabPer = kPenCap / 32;             // table entries per producer lane
constexpr int kMaxRowStages = 48;                 // rows up to 1.5 MB
constexpr int kFlagWords = kMaxRowStages * kStrThreads / 32;
constexpr int kSlotKeys = 512;                    // a handed-over row's keys: survivors and table columns
constexpr int kHash = 2 * kPenCap;                // flagged streaming threads' element masks (open addressing)
constexpr uint32_t kHashEmpty = 0xFFFFFFFFu;
enum : int { kEndSelectors = 0, kEndFinisher = 1 };
static_assert(kStageVecs % kThreads == 0 && kStageVecs == kStrThreads * kVecPerThread, "stage split");
static_assert(kSelVecs * 8 <= 64, "one 64-bit survivor mask per selector thread and stage");
static_assert(kVecPerThread * 8 <= 32, "one 32-bit element mask per streaming thread and stage");

// Per-slot block: record, published and final streamer partials, penalty table and flags.
struct Slot {
  int rec[kMetaWords];
  float lse_w[kStrWarps];       // streaming warp w: log-sum-exp of its columns so far
  float part_m[kStrWarps];      // final (max, sum) partial per streaming warp
  float part_s[kStrWarps];
  int pen_n;                    // entries in the table
  uint32_t lse_ord;             // ord of the log-sum-exp over the 16 published values: a lower bound of
                                // the row's lse (raised with atomicMax, so it never goes down)
  int stages_done;              // stages whose combined bound lse_ord covers
  uint32_t kcnt;                // rows started with the request's bound: survivors reserved in `keys`
  int kovf;                     // such a row's survivors did not all fit `keys` (the selectors end it)
  int kfail;                    // the first reservation that did not fit: keys [0, kfail) are written
  int end_by;                   // kEndSelectors / kEndFinisher
  int pad[25];
  int sprog[kMaxRowStages];     // streaming warps that have published each stage
  int tab_tok[kPenCap];         // penalised local columns
  float tab_y[kPenCap];         // their processed values
  uint32_t flags[kFlagWords];   // bit stage * kStrThreads + t: streaming thread t's vectors of that stage hold one
  uint32_t hkey[kHash];         // such a (stage * kStrThreads + t), or kHashEmpty
  uint32_t hmask[kHash];   // its bit j * EPV + e: element e of the thread's vector j is penalised
  unsigned long long keys[kSlotKeys];   // value keys ord(y) | ~flat of those rows
};

constexpr size_t kOffSlots = kOffWin;
constexpr size_t kSlotBytes = align128(sizeof(Slot));
constexpr size_t kOffRowBars = kOffSlots + kSlots * kSlotBytes;
constexpr size_t kOffFlags = kOffRowBars + align128(4 * kSlots * 8);
constexpr size_t kOffRing = kOffFlags + 128;

__host__ __device__ constexpr size_t smem_bytes(int stages) { return kOffRing + size_t(stages) * kStage; }
static_assert(smem_bytes(5) <= 227 * 1024, "five ring stages fit one CTA's shared memory");

struct View {
  Slot* slot0;
  uint64_t* recfull;   // [kSlots] producer -> streamers, selectors: record and penalty table written
  uint64_t* rowdone;   // [kSlots] streamers -> selectors: final partials (one arrival per streaming warp)
  uint64_t* findone;   // [kSlots] finisher -> producer: slot free
  uint64_t* handoff;   // [kSlots] selectors -> finisher: the row's candidate pass is over (end_by says who ends it)
  volatile int* sel_abort;   // [kSlots] selectors' per-row abort decision
  unsigned char* ring;
  __device__ __forceinline__ Slot* slot(int q) const {
    return reinterpret_cast<Slot*>(reinterpret_cast<unsigned char*>(slot0) + q * kSlotBytes);
  }
};

__device__ __forceinline__ View view() {
  View W;
  W.slot0 = reinterpret_cast<Slot*>(g_smem + kOffSlots);
  W.recfull = reinterpret_cast<uint64_t*>(g_smem + kOffRowBars);
  W.rowdone = W.recfull + kSlots;
  W.findone = W.recfull + 2 * kSlots;
  W.handoff = W.recfull + 3 * kSlots;
  W.sel_abort = reinterpret_cast<volatile int*>(g_smem + kOffFlags);
  W.ring = g_smem + kOffRing;
  return W;
}

// Table entry of local column tl, or -1 (a scan: at most kPenCap entries).
__device__ __forceinline__ int table_find(const Slot* sl, int tl) {
  for (int j = 0; j < sl->pen_n; ++j)
    if (sl->tab_tok[j] == tl) return j;
  return -1;
}

__device__ __forceinline__ uint32_t hash_of(uint32_t key) { return (key * 2654435761u) >> 24; }
static_assert(kHash == 256, "hash_of gives 8 bits");

// Add `bits` to the mask of flagged thread `key` (producer; at most kPenCap
// keys in kHash places, so a place is always found).
__device__ __forceinline__ void hash_add(Slot* sl, uint32_t key, uint32_t bits) {
  uint32_t h = hash_of(key);
  for (int p = 0; p < kHash; ++p) {
    const uint32_t old = atomicCAS(&sl->hkey[h], kHashEmpty, key);
    if (old == kHashEmpty || old == key) {
      atomicOr(&sl->hmask[h], bits);
      return;
    }
    h = (h + 1) & (kHash - 1);
  }
}

// The element mask of flagged thread `key` (0 when absent).
__device__ __forceinline__ uint32_t hash_find(const Slot* sl, uint32_t key) {
  uint32_t h = hash_of(key);
  for (int p = 0; p < kHash; ++p) {
    const uint32_t k = sl->hkey[h];
    if (k == key) return sl->hmask[h];
    if (k == kHashEmpty) return 0u;
    h = (h + 1) & (kHash - 1);
  }
  return 0u;
}

// The streamers publish their lse bound after stages 0, 2, 6, 14, 30 (a row's
// stages 2^k - 2: the bound grows fastest early in the row, and every
// publication is the streaming warps' longest chain; publishing after every
// second or fourth stage, or after 0, 1, 3, 7, 15, measured slower).
__host__ __device__ constexpr bool published(int ch) { return ((ch + 2) & (ch + 1)) == 0; }
// The last published stage at or before stage ch (rows have at most kMaxRowStages <= 62 stages).
__host__ __device__ constexpr int last_published(int ch) {
  return ch >= 30 ? 30 : ch >= 14 ? 14 : ch >= 6 ? 6 : ch >= 2 ? 2 : 0;
}
static_assert(kMaxRowStages <= 62, "last_published covers every stage index");
static_assert(published(0) && !published(1) && last_published(1) == 0 && last_published(5) == 2 &&
              last_published(13) == 6 && last_published(29) == 14 && published(last_published(47)), "publication");

// The published lower bound of a slot's row lse (-inf when none).
__device__ __forceinline__ float lse_bound_of(const Slot* sl) {
  const float v = ord_to_f32(*reinterpret_cast<const volatile uint32_t*>(&sl->lse_ord));
  return (v > -kInf && v < kInf) ? v : -kInf;
}

__host__ __device__ __forceinline__ bool pen_used(const Params& P) {
  return P.pen && P.T > 0 && P.mode == kModeProcessed;
}
}  // namespace sel

// Penalty tables, one warp per row: the distinct history tokens of an
// unconstrained row that this shard holds, in order of first occurrence, as
// local columns with their processed values (vLLM apply_penalties over the
// output history, then the temperature); valid entries first, -1 after.
// Launched between the row metadata kernel and the selecting kernel.
template <typename TL>
__global__ void __launch_bounds__(256) pen_table_kernel(const __grid_constant__ Params P) {
  pdl_trigger();
  // the histories and node ids may come from the previous step's merge, which
  // the row records kernel waits for: wait for that grid before reading
  pdl_wait();
  constexpr int ES = sizeof(TL);
  const int lane = lane_id();
  const int row = static_cast<int>(blockIdx.x) * (256 / 32) + warp_id();
  if (row < P.R * P.NB) {
    const int r = row / P.NB;
    int* dst = P.pen_tab + static_cast<size_t>(row) * 2 * P.tabw;
    const float rep = P.rep ? P.rep[r] : 1.0f;
    const float pres = P.pres ? P.pres[r] : 0.0f;
    const float freq = P.freq ? P.freq[r] : 0.0f;
    int n_tab = 0;
    if (P.node[row] == GR_NODE_UNCONSTRAINED && !(rep == 1.0f && pres == 0.0f && freq == 0.0f)) {
      const float teff = eff_temperature(P, r);
      const int* h = P.hist + static_cast<size_t>(row) * P.T;
      const TL* rowp = reinterpret_cast<const TL*>(row_geom<ES, sel::kStage>(P, row).rowp);
      // the history in registers (T <= kPenCap: four tokens per lane), counted
      // by shuffles; the penalised columns' logits loaded before any is used
      constexpr int kPer = sel::kTabPer;
      int tk[kPer], cnt[kPer], first[kPer];
#pragma unroll
      for (int k = 0; k < kPer; ++k) {
        tk[k] = (k * 32 + lane < P.T) ? h[k * 32 + lane] : -1;
        cnt[k] = 0;
        first[k] = 1;
      }
      const int groups = (P.T + 31) / 32;   // register groups that hold history tokens
#pragma unroll
      for (int kk = 0; kk < kPer; ++kk) {
        for (int j = 0; j < 32 && kk * 32 + j < P.T; ++j) {   // position kk * 32 + j, uniform bounds
          const int o = __shfl_sync(0xFFFFFFFFu, tk[kk], j);
#pragma unroll
          for (int k = 0; k < kPer; ++k) {
            if (k < groups) {
              cnt[k] += (o == tk[k]);
              if (kk * 32 + j < k * 32 + lane && o == tk[k]) first[k] = 0;
            }
          }
        }
      }
      int col[kPer];
      float xr[kPer];
#pragma unroll
      for (int k = 0; k < kPer; ++k) {
        col[k] = (tk[k] >= 0 && first[k]) ? col_of(P, tk[k]) : -1;
        xr[k] = (col[k] >= 0) ? LogitTraits<TL>::load1(rowp + col[k]) : 0.0f;
      }
#pragma unroll
      for (int k = 0; k < kPer; ++k) {
        const bool mine = col[k] >= 0;
        const unsigned ball = __ballot_sync(0xFFFFFFFFu, mine);
        const int idx = n_tab + __popc(ball & ((1u << lane) - 1u));
        if (mine && idx < P.tabw) {
          const float xp = penalise(xr[k], cnt[k], rep, pres, freq);
          dst[idx] = col[k];
          dst[P.tabw + idx] = __float_as_int((teff == 1.0f) ? xp : __fdiv_rn(xp, teff));
        }
        n_tab += __popc(ball);
      }
    }
    for (int i = min(n_tab, P.tabw) + lane; i < P.tabw; i += 32) dst[i] = -1;
  }
}

// Producer warp: per row its record, its penalty table and flags, then its body.
template <typename TL>
__device__ void sel_produce(const Params& P) {
  constexpr int ES = sizeof(TL);
  constexpr int EPV = LogitTraits<TL>::kPerVec;
  const Smem S = smem_view(P);
  const sel::View W = sel::view();
  const int lane = lane_id();
  const uint64_t pol = l2_policy_evict_first();
  int stage = 0;
  uint32_t round = 0;
  long long fills = 0;
  const int total = P.R * P.NB;
  auto draw = [&]() -> int {
    int seq = 0;
    if (lane == 0) seq = static_cast<int>(atomicAdd(P.row_counter, 1u));
    seq = __shfl_sync(0xFFFFFFFFu, seq, 0);
    return (seq < total) ? row_of_seq(P, seq) : -1;
  };
  // the next row's record word, request bound and table entries, loaded a row ahead
  int meta_word = 0;
  unsigned long long tau_word = 0;
  int tk_n[sel::kTabPer], ty_n[sel::kTabPer];
  auto fetch = [&](int row) {
#pragma unroll
    for (int k = 0; k < sel::kTabPer; ++k) {
      tk_n[k] = -1;
      ty_n[k] = 0;
    }
    if (row < 0) return;
    meta_word = __ldcg(P.meta + static_cast<size_t>(row) * kMetaWords + lane);
    if (lane == 0) tau_word = ld_relaxed_u64(P.tau + row / P.NB);
    if (P.pen_tab != nullptr) {
      const int* tb = P.pen_tab + static_cast<size_t>(row) * 2 * P.tabw;
#pragma unroll
      for (int k = 0; k < sel::kTabPer; ++k) {
        if (k * 32 < P.tabw) {
          tk_n[k] = __ldcg(tb + k * 32 + lane);
          ty_n[k] = __ldcg(tb + P.tabw + k * 32 + lane);
        }
      }
    }
  };
  int row_next = draw();
  fetch(row_next);
  SEL_T(t_prod);
  for (int it = 0;; ++it) {
    const int q = it % sel::kSlots;
    sel::Slot* sl = W.slot(q);
    const int row = row_next;
    SEL_T(t_fd);
    if (it >= sel::kSlots) {
      int good = 1;
      if (lane == 0)
        good = mbar_wait_bounded(&W.findone[q], static_cast<uint32_t>(it / sel::kSlots - 1) & 1u, &S.v->abort) ? 1 : 0;
      if (!__shfl_sync(0xFFFFFFFFu, good, 0)) {
        if (lane == 0) {
          if (!S.v->abort) atomicOr(P.err, GR_DEVERR_TIMEOUT);
          S.v->abort = 1;
        }
        break;
      }
    }
    if (row < 0) {
      if (lane == 0) {
        sl->rec[kMRow] = -1;
        mbar_arrive(&W.recfull[q]);
      }
      break;
    }
    SEL_ADD(lane == 0, 7, t_fd);
    const int cur = meta_word;
    const unsigned long long tau_cur = __shfl_sync(0xFFFFFFFFu, tau_word, 0);
    int tk[sel::kTabPer], ty[sel::kTabPer];
#pragma unroll
    for (int k = 0; k < sel::kTabPer; ++k) {
      tk[k] = tk_n[k];
      ty[k] = ty_n[k];
    }
    sl->rec[lane] = (lane == kMTauLo) ? static_cast<int>(tau_cur & 0xFFFFFFFFull)
                  : (lane == kMTauHi) ? static_cast<int>(tau_cur >> 32) : cur;
    row_next = draw();
    fetch(row_next);
    // the slot's state starts empty for the new row
    for (int w = lane; w < sel::kFlagWords; w += 32) sl->flags[w] = 0u;
    for (int w = lane; w < sel::kMaxRowStages; w += 32) sl->sprog[w] = 0;
    for (int w = lane; w < sel::kHash; w += 32) {
      sl->hkey[w] = sel::kHashEmpty;
      sl->hmask[w] = 0u;
    }
    if (lane < sel::kStrWarps) sl->lse_w[lane] = -kInf;
    if (lane == 0) {
      sl->lse_ord = f32_to_ord(-kInf);
      sl->stages_done = 0;
      sl->kcnt = 0u;
      sl->kovf = 0;
      sl->kfail = sel::kSlotKeys;
      sl->end_by = sel::kEndSelectors;
    }
    __syncwarp();   // the flags are zero before any lane sets one
    // the penalty table and the flag of the streaming thread whose vectors hold each entry
    int n_tab = 0;
    if (P.pen_tab != nullptr) {
      const Geom g = row_geom<ES, sel::kStage>(P, row);
#pragma unroll
      for (int k = 0; k < sel::kTabPer; ++k) {
        const bool v = tk[k] >= 0;
        const unsigned ball = __ballot_sync(0xFFFFFFFFu, v);
        if (v) {
          const int idx = n_tab + __popc(ball & ((1u << lane) - 1u));
          sl->tab_tok[idx] = tk[k];
          sl->tab_y[idx] = __int_as_float(ty[k]);
          if (tk[k] >= g.head && tk[k] < g.tail_start) {
            const int gv = (tk[k] - g.head) / EPV;               // body vector
            const int e = (tk[k] - g.head) - gv * EPV;           // its element
            const int st = gv / sel::kStageVecs;
            const int vs = gv - st * sel::kStageVecs;             // vector within the stage
            const int t_str = vs % sel::kStrThreads;              // streaming thread and its vector j
            const int j = vs / sel::kStrThreads;
            const int bit = st * sel::kStrThreads + t_str;
            if (st < sel::kMaxRowStages) {
              atomicOr(&sl->flags[bit >> 5], 1u << (bit & 31));
              sel::hash_add(sl, static_cast<uint32_t>(bit), 1u << (j * EPV + e));
            }
          }
        }
        n_tab += __popc(ball);
      }
    }
    if (lane == 0) sl->pen_n = n_tab;
    __syncwarp();
    int ok = 1;
    if (lane == 0) {
      mbar_arrive(&W.recfull[q]);   // release: record, bounds, table and flags
      const Geom g = row_geom<ES, sel::kStage>(P, row);
      for (int ch = 0; ch < (P.stall_copies ? 0 : g.nchunks); ++ch) {
        if (fills >= P.stages && !mbar_wait_bounded(&S.empty[stage], (round - 1u) & 1u, &S.v->abort)) {
          if (!S.v->abort) atomicOr(P.err, GR_DEVERR_TIMEOUT);
          S.v->abort = 1;
          ok = 0;
          break;
        }
        const long long off = static_cast<long long>(ch) * sel::kStage;
        const uint32_t bytes = static_cast<uint32_t>(min(static_cast<long long>(sel::kStage), g.body_bytes - off));
        fence_proxy_async_smem();
        mbar_arrive_expect_tx(&S.full[stage], bytes);
        bulk_copy_g2s(W.ring + static_cast<size_t>(stage) * sel::kStage, g.body + off, bytes, &S.full[stage], pol);
        ++fills;
        if (++stage == P.stages) {
          stage = 0;
          ++round;
        }
      }
    }
    if (!__shfl_sync(0xFFFFFFFFu, ok, 0)) break;
  }
  SEL_ADD(lane == 0, 15, t_prod);
  if (lane == 0) {
    S.v->issued = fills;
    __threadfence_block();
    S.v->producer_done = 1;
  }
}

// Lower bound of the row's lse from the streaming warps' published values
// (stale ones are still lower bounds; -inf when none is known).
__device__ __forceinline__ float sel_lse_bound(const sel::Slot* sl) {
  float lw[sel::kStrWarps];
  float mx = -kInf;
#pragma unroll
  for (int w = 0; w < sel::kStrWarps; ++w) {
    const float v = *reinterpret_cast<const volatile float*>(&sl->lse_w[w]);
    lw[w] = (v > -kInf && v < kInf) ? v : -kInf;
    mx = fmaxf(mx, lw[w]);
  }
  if (!(mx > -kInf)) return -kInf;
  float t = 0.0f;
#pragma unroll
  for (int w = 0; w < sel::kStrWarps; ++w) t += fast_exp2((lw[w] - mx) * kLog2e);
  return mx + __logf(t);
}

// Streamers: (max, sum exp) of every row, penalised columns left out; after
// each stage the warp's log-sum-exp so far goes to the slot, and the stage's
// last warp combines the sixteen into lse_ord before counting the stage done.
// Only the stages the selectors read a bound after are published (0, 2, 6, 14,
// 30): the publication is the streamers' longest chain.
template <typename TL>
__device__ void sel_stream_rows(const Params& P) {
  const Smem S = smem_view(P);
  const sel::View W = sel::view();
  using Tr = LogitTraits<TL>;
  constexpr int ES = sizeof(TL);
  constexpr int EPV = Tr::kPerVec;
  constexpr int kVPT = sel::kVecPerThread;
  const int sid = static_cast<int>(threadIdx.x) - sel::kSelWarps * 32;
  const int swarp = sid >> 5, lane = lane_id();
  int cstage = 0;
  uint32_t cphase = 0;
  long long consumed = 0;
  bool aborted = false;
  SEL_T(t_str);
  for (int it = 0;; ++it) {
    const int q = it % sel::kSlots;
    sel::Slot* sl = W.slot(q);
    if (!mbar_wait_bounded(&W.recfull[q], static_cast<uint32_t>(it / sel::kSlots) & 1u, &S.v->abort)) {
      if (!S.v->abort) atomicOr(P.err, GR_DEVERR_TIMEOUT);
      S.v->abort = 1;
    }
    if (__any_sync(0xFFFFFFFFu, S.v->abort != 0)) {
      aborted = true;
      break;
    }
    const int row = sl->rec[kMRow];
    if (row < 0) break;
    const float yscale = (P.mode == kModeProcessed) ? __int_as_float(sl->rec[kMRteff]) : 1.0f;
    const float a = kLog2e * yscale;
    const int pen_n = sl->pen_n;
    float m = -kInf, s = 0.0f;
    const Geom g = row_geom<ES, sel::kStage>(P, row);
    {
      const int nh = g.head, nt = P.VL - g.tail_start;
      const TL* rowp = reinterpret_cast<const TL*>(g.rowp);
      for (int i = sid; i < nh + nt; i += sel::kStrThreads) {
        const int tl = (i < nh) ? i : g.tail_start + (i - nh);
        if (pen_n > 0 && sel::table_find(sl, tl) >= 0) continue;   // its value comes from the table
        const float y = Tr::load1(rowp + tl) * yscale;
        if (y > m) {
          s = s * fast_exp2((m - y) * kLog2e);
          m = y;
        }
        if (m > -kInf) s += fast_exp2((y - m) * kLog2e);
      }
    }
    uint64_t sacc0 = pack2(0.0f, 0.0f), sacc1 = pack2(0.0f, 0.0f);
    for (int ch = 0; ch < g.nchunks; ++ch) {
      SEL_T(t_sw);
      if (!mbar_wait_bounded(&S.full[cstage], cphase, &S.v->abort)) {
        if (!S.v->abort) atomicOr(P.err, GR_DEVERR_TIMEOUT);
        S.v->abort = 1;
      }
      SEL_ADD(sid == 0, 10, t_sw);
      const long long off = static_cast<long long>(ch) * sel::kStage;
      const int nvec = static_cast<int>(min(static_cast<long long>(sel::kStage), g.body_bytes - off) >> 4);
      const uint4* sv = reinterpret_cast<const uint4*>(W.ring + static_cast<size_t>(cstage) * sel::kStage);
      uint4 vv[kVPT];
#pragma unroll
      for (int j = 0; j < kVPT; ++j)
        vv[j] = (sid + j * sel::kStrThreads < nvec) ? sv[sid + j * sel::kStrThreads] : make_uint4(0, 0, 0, 0);
      __syncwarp();
      if (lane == 0) mbar_arrive(&S.empty[cstage]);
      if (++cstage == P.stages) {
        cstage = 0;
        cphase ^= 1u;
      }
      ++consumed;
      // penalised columns among this thread's vectors of the stage: -inf in the sum
      const int bit = ch * sel::kStrThreads + sid;
      if (pen_n > 0 && ch < sel::kMaxRowStages && ((sl->flags[bit >> 5] >> (bit & 31)) & 1u)) {
        const uint32_t pmask = sel::hash_find(sl, static_cast<uint32_t>(bit));
#pragma unroll
        for (int j = 0; j < kVPT; ++j) {
          const uint32_t fl = (pmask >> (j * EPV)) & ((1u << EPV) - 1u);
          if (fl && sid + j * sel::kStrThreads < nvec) Tr::mask_neg_inf(vv[j], fl);
        }
      }
      if (m == -kInf) {
        // the running reference: any finite value of the thread's first vectors
        float mx = -kInf;
#pragma unroll
        for (int j = 0; j < kVPT; ++j) {
          if (sid + j * sel::kStrThreads < nvec) {
            float x[EPV];
            Tr::unpack(vv[j], x);
#pragma unroll
            for (int e = 0; e < EPV; ++e) mx = fmaxf(mx, x[e]);
          }
        }
        m = (mx > -kInf && mx < kInf) ? mx * yscale : -kInf;
      }
      if (m > -kInf) {
        const float cm = -m * kLog2e;
        const uint64_t A2 = pack2(a, a), C2 = pack2(cm, cm);
#pragma unroll
        for (int j = 0; j < kVPT; ++j)
          if (sid + j * sel::kStrThreads < nvec) FastSum<TL>::add(vv[j], A2, C2, sacc0, sacc1);
      }
      // publish the warp's log-sum-exp so far at the stages the selectors read
      // (stages 0, 2, 6, 14, 30), then count the stage as published
      if (sel::published(ch)) {
        float q0, q1, q2, q3;
        unpack2(sacc0, q0, q1);
        unpack2(sacc1, q2, q3);
        float t = s + ((q0 + q1) + (q2 + q3));
        float M = m;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) M = fmaxf(M, __shfl_xor_sync(0xFFFFFFFFu, M, o));
        t = (m == -kInf) ? 0.0f : t * fast_exp2((m - M) * kLog2e);
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) t += __shfl_xor_sync(0xFFFFFFFFu, t, o);
        const float lw = (M > -kInf && t > 0.0f && t < kInf) ? M + __logf(t) : -kInf;
        if (lane == 0) {
          *reinterpret_cast<volatile float*>(&sl->lse_w[swarp]) = lw;
          __threadfence_block();
          // (a row has at most kMaxRowStages stages: the launch checks it)
          if (ch < sel::kMaxRowStages && atomicAdd(&sl->sprog[ch], 1) + 1 == sel::kStrWarps) {
            // the stage's last warp: the combined bound, then the stage count
            // waited on (in this order)
            atomicMax(&sl->lse_ord, f32_to_ord(sel_lse_bound(sl)));
            __threadfence_block();
            atomicMax(&sl->stages_done, ch + 1);
          }
        }
      }
    }
    fold(sacc0, sacc1, s);
    float M = m;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) M = fmaxf(M, __shfl_xor_sync(0xFFFFFFFFu, M, o));
    s = (m == -kInf) ? 0.0f : s * fast_exp2((m - M) * kLog2e);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xFFFFFFFFu, s, o);
    if (lane == 0) {
      sl->part_m[swarp] = M;
      sl->part_s[swarp] = s;
      mbar_arrive(&W.rowdone[q]);   // release: the warp's final partial
    }
  }
  SEL_ADD(sid == 0, 11, t_str);
  if (aborted && sid == 0) {
    // wait (bounded) for the producer to stop and for its copies still in flight
    const uint64_t t0 = global_timer_ns();
    while (!*reinterpret_cast<volatile int*>(&S.v->producer_done) && global_timer_ns() - t0 < kWaitLimitNs) {
    }
    const long long issued = *reinterpret_cast<volatile long long*>(&S.v->issued);
    for (long long c = consumed; c < issued; ++c) {
      mbar_wait_bounded(&S.full[cstage], cphase);
      if (++cstage == P.stages) {
        cstage = 0;
        cphase ^= 1u;
      }
    }
  }
}

// Exact log-sum-exp of a row from global memory (two passes), the penalised
// columns with their table values, for rows whose streamed sum was not finite.
// Selector threads only.
template <typename TL>
__device__ float sel_exact_row_lse(const Params& P, const RowCtx& c, const Step<TL, true>& st,
                                   const sel::Slot* sl) {
  const Smem S = smem_view(P);
  const int tid = threadIdx.x, lane = lane_id(), warp = warp_id();
  const float ys = (P.mode == kModeProcessed) ? c.rteff : 1.0f;
  const int pen_n = sl->pen_n;
  auto yval = [&](int i) -> float {
    const int j = (pen_n > 0) ? sel::table_find(sl, i) : -1;
    return (j >= 0) ? sl->tab_y[j] : st.load_logit(c, i) * ys;
  };
  float mx = -kInf;
  for (int i = tid; i < P.VL; i += kThreads) mx = fmaxf(mx, yval(i));
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xFFFFFFFFu, mx, o));
  if (lane == 0) S.red_m[warp] = mx;
  csync();
  float M = -kInf;
#pragma unroll
  for (int w = 0; w < kWarps; ++w) M = fmaxf(M, S.red_m[w]);
  float sm = 0.0f;
  if (M > -kInf)
    for (int i = tid; i < P.VL; i += kThreads) sm += fast_exp2((yval(i) - M) * kLog2e);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) sm += __shfl_xor_sync(0xFFFFFFFFu, sm, o);
  if (lane == 0) S.red_s[warp] = sm;
  csync();
  float tot = 0.0f;
#pragma unroll
  for (int w = 0; w < kWarps; ++w) tot += S.red_s[w];
  csync();
  return (M == -kInf) ? -kInf : M + logf(tot);
}

// Selectors: the candidate pass of every stage and the row end.
template <typename TL>
__device__ void sel_select_rows(const Params& P) {
  const Smem S = smem_view(P);
  const sel::View W = sel::view();
  Step<TL, true> st(P);
  using Tr = LogitTraits<TL>;
  constexpr int ES = sizeof(TL);
  constexpr int EPV = Tr::kPerVec;
  const int tid = threadIdx.x, lane = lane_id();
  int cstage = 0;
  uint32_t cphase = 0;
  SEL_T(t_sel);
  for (int it = 0;; ++it) {
    const int q = it % sel::kSlots;
    const uint32_t par = static_cast<uint32_t>(it / sel::kSlots) & 1u;
    sel::Slot* sl = W.slot(q);
    bool ok = mbar_wait_bounded(&W.recfull[q], par, &S.v->abort);
    if (!ok) {
      if (!S.v->abort) atomicOr(P.err, GR_DEVERR_TIMEOUT);
      S.v->abort = 1;
    }
    // one decision for every selector: no record (the streamers drain the
    // copies in flight) or the stop record ends the loop for all
    csync();
    if (tid == 0) W.sel_abort[q] = (S.v->abort || sl->rec[kMRow] < 0) ? 1 : 0;
    csync();
    if (W.sel_abort[q]) break;
    RowCtx c;
    const int* rec = sl->rec;
    c.row = rec[kMRow];
    c.r = rec[kMR];
    c.b = rec[kMB];
    fill_row_ctx<TL>(P, rec, c);
    st.rec = rec;
    st.ext_tok = sl->tab_tok;
    st.ext_y = sl->tab_y;
    st.ext_n = &sl->pen_n;
    const int pen_n = sl->pen_n;
    const float yscale = (P.mode == kModeProcessed) ? c.rteff : 1.0f;
    if (tid == 0) {
      S.v->abort_snap = S.v->abort;                   // one decision for every selector
      const uint64_t tau_pref = static_cast<uint64_t>(static_cast<uint32_t>(rec[kMTauLo])) |
                                (static_cast<uint64_t>(static_cast<uint32_t>(rec[kMTauHi])) << 32);
      S.v->cnt = 0;
      S.v->overflow = 0;
      S.v->discard = 0;
      S.v->tau_pref = tau_pref;
      S.v->thr_key = 0ull;
      S.v->thr_y = -kInf;
      if (P.eos_score) P.eos_score[c.row] = __int_as_float(0x7FC00000);
    }
    csync();
    const bool cand = c.stream && !S.v->abort_snap;   // rows with a candidate pass (dead rows have none)
    uint64_t tau_seen = S.v->tau_pref;
    bool fast = tau_seen != 0ull;                     // the request has a bound (the same value everywhere)
    // a row that starts with the bound keeps its few survivors in its slot,
    // for the finisher; the others in the selectors' list
    const bool in_slot = fast;
    uint64_t* const kbuf = in_slot ? reinterpret_cast<uint64_t*>(sl->keys) : S.keys;
    uint32_t* const kcnt = in_slot ? &sl->kcnt : &S.v->cnt;
    const uint32_t kcap = in_slot ? static_cast<uint32_t>(sel::kSlotKeys) : static_cast<uint32_t>(kKeyCap);
    float thr_y = -kInf;
    const Geom g = row_geom<ES, sel::kStage>(P, c.row);
    const uint32_t vb = static_cast<uint32_t>(c.b) * static_cast<uint32_t>(P.V);
    // head / tail columns outside the bulk-copied body: candidates as they are
    if (cand) {
      const int nh = g.head, nt = P.VL - g.tail_start;
      for (int ib = 0; ib < nh + nt; ib += kThreads) {
        const int i = ib + tid;
        bool pred = false;
        uint64_t key = 0ull;
        if (i < nh + nt) {
          const int tl = (i < nh) ? i : g.tail_start + (i - nh);
          if (!(pen_n > 0 && sel::table_find(sl, tl) >= 0)) {
            const float x = st.load_logit(c, tl);
            const float ye = (P.mode == kModeProcessed && c.teff != 1.0f) ? __fdiv_rn(x, c.teff) : x;
            key = make_key(ye, vb + static_cast<uint32_t>(tok_of(P, tl)));
            pred = true;
          }
        }
        warp_append(pred, key, kbuf, kcnt, kcap, &S.v->overflow);
      }
      csync();
    }
    // shrink the row's list to its best kk keys; the kk-th bounds the rest of the row
    auto shrink_row = [&]() {
      const Cut cut = st.shrink_to(P.kk);
      if (tid == 0) {
        S.v->discard = 1;
        S.v->thr_key = cut.floor_key();
        const float ty = key_score(cut.floor_key());
        S.v->thr_y = ty - fabsf(ty) * 2.0e-6f - 1e-30f;
      }
      csync();
      thr_y = S.v->thr_y;
    };
    for (int ch = 0; ch < g.nchunks; ++ch) {
      SEL_T(t_fw);
      if (!mbar_wait_bounded(&S.full[cstage], cphase, &S.v->abort)) {
        if (!S.v->abort) atomicOr(P.err, GR_DEVERR_TIMEOUT);
        S.v->abort = 1;
      }
      SEL_ADD(tid == 0, 1, t_fw);
      const long long off = static_cast<long long>(ch) * sel::kStage;
      const int nvec = static_cast<int>(min(static_cast<long long>(sel::kStage), g.body_bytes - off) >> 4);
      const unsigned char* stage_p = W.ring + static_cast<size_t>(cstage) * sel::kStage;
      const uint4* sv = reinterpret_cast<const uint4*>(stage_p);
      if (cand) {
        // the streamers' bound covers a stage once its last streaming warp has
        // combined it: a row's first stage (and every stage before the request
        // has a bound) waits for that, bounded
        SEL_T(t_pw);
        if (ch == 0 || !fast) {
          const int need = sel::last_published(ch) + 1;
          const uint64_t t0 = global_timer_ns();
          while (*reinterpret_cast<volatile int*>(&sl->stages_done) < need) {
            if (*reinterpret_cast<volatile int*>(&S.v->abort)) break;
            if (global_timer_ns() - t0 > kWaitLimitNs) {
              if (!S.v->abort) atomicOr(P.err, GR_DEVERR_TIMEOUT);
              S.v->abort = 1;
              break;
            }
            __nanosleep(64);
          }
          __threadfence_block();   // the bound is read after its stage count
        }
        SEL_ADD(tid == 0, 0, t_pw);
        SEL_T(t_scan);
        // the floor: the request bound as read one stage earlier, through the
        // streamers' lower bound of the row's lse
        const uint64_t tau_use = tau_seen;
        tau_seen = ld_relaxed_u64(P.tau + c.r);
        const float floor_y = st.tau_floor(c, tau_use, sel::lse_bound_of(sl));
        const float thr_e = fmaxf(thr_y, floor_y);
        const int tbase = g.head + ch * sel::kStageVecs * EPV;
        // survivors: bit j * EPV + e for element e of vector j (j < kSelVecs);
        // the vectors in batches of four, loaded together and tested by their
        // common maximum first
        uint64_t pm = 0;
#pragma unroll
        for (int jb = 0; jb < sel::kSelVecs; jb += 4) {
          uint4 w[4];
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            const int v = tid + (jb + j) * kThreads;
            w[j] = (v < nvec) ? sv[v] : make_uint4(0, 0, 0, 0);
          }
          float bm = -kInf;
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            float x[EPV];
            Tr::unpack(w[j], x);
#pragma unroll
            for (int e = 0; e < EPV; ++e) bm = fmaxf(bm, x[e]);
          }
          if (bm * yscale >= thr_e) {
#pragma unroll
            for (int j = 0; j < 4; ++j) {
              const int v = tid + (jb + j) * kThreads;
              if (v < nvec) {
                float x[EPV];
                Tr::unpack(w[j], x);
                float vmax = x[0];
#pragma unroll
                for (int e = 1; e < EPV; ++e) vmax = fmaxf(vmax, x[e]);
                if (vmax * yscale >= thr_e) {
                  uint32_t fl = 0;
                  const int sbit = ch * sel::kStrThreads + (v % sel::kStrThreads);
                  if (pen_n > 0 && ch < sel::kMaxRowStages && ((sl->flags[sbit >> 5] >> (sbit & 31)) & 1u))
                    fl = (sel::hash_find(sl, static_cast<uint32_t>(sbit)) >> ((v / sel::kStrThreads) * EPV)) &
                         ((1u << EPV) - 1u);
#pragma unroll
                  for (int e = 0; e < EPV; ++e)
                    if (!((fl >> e) & 1u) && x[e] * yscale >= thr_e) pm |= 1ull << ((jb + j) * EPV + e);
                }
              }
            }
          }
        }
        const uint32_t cl = static_cast<uint32_t>(__popcll(pm));
        if (fast) {
          // the request has a bound: survivors are few; each warp reserves
          // and writes its own, with no barrier.  A reservation that does not
          // fit marks the row, which is then selected exactly at its end.
          if (__any_sync(0xFFFFFFFFu, cl != 0)) {
            uint32_t inc = cl;
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
              const uint32_t t = __shfl_up_sync(0xFFFFFFFFu, inc, o);
              if (lane >= o) inc += t;
            }
            const uint32_t wtot = __shfl_sync(0xFFFFFFFFu, inc, 31);
            uint32_t base = 0;
            if (lane == 31) base = atomicAdd(kcnt, wtot);
            SEL_CNT(lane == 31, 14, wtot);
            base = __shfl_sync(0xFFFFFFFFu, base, 31);
            uint64_t* dst = kbuf;
            bool fits = base + wtot <= kcap;
            if (!fits && in_slot) {
              // the slot is full (a weak bound): the row's further survivors go
              // to the selectors' list, and the selectors end the row
              if (lane == 31) {
                atomicMin(&sl->kfail, static_cast<int>(base));
                sl->kovf = 1;
                base = atomicAdd(&S.v->cnt, wtot);
              }
              base = __shfl_sync(0xFFFFFFFFu, base, 31);
              dst = S.keys;
              fits = base + wtot <= static_cast<uint32_t>(kKeyCap);
            }
            if (fits) {
              uint32_t pos = base + inc - cl;
              uint64_t mk = pm;
              while (mk) {
                const int bi = __ffsll(static_cast<long long>(mk)) - 1;
                mk &= mk - 1ull;
                const int col = (tid + (bi / EPV) * kThreads) * EPV + (bi % EPV);
                const float x = Tr::load_s(stage_p, col);
                const float ye = (P.mode == kModeProcessed && c.teff != 1.0f) ? __fdiv_rn(x, c.teff) : x;
                dst[pos++] = make_key(ye, vb + static_cast<uint32_t>(tok_of(P, tbase + col)));
              }
            } else if (lane == 0) {
              *reinterpret_cast<volatile int*>(&S.v->overflow) = 1;   // the row is read again exactly
            }
          }
          SEL_ADD(tid == 0, 2, t_scan);
        } else {
          // no request bound yet: the row keeps its own (its kk-th key), which
          // needs the list's length between barriers
          uint32_t inc = 0, base = 0, wtot = 0;
          if (__any_sync(0xFFFFFFFFu, cl != 0)) {
            inc = cl;
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
              const uint32_t t = __shfl_up_sync(0xFFFFFFFFu, inc, o);
              if (lane >= o) inc += t;
            }
            wtot = __shfl_sync(0xFFFFFFFFu, inc, 31);
            if (lane == 31) base = atomicAdd(&S.v->cnt, wtot);
            base = __shfl_sync(0xFFFFFFFFu, base, 31);
          }
          csync();
          const bool fits = S.v->cnt <= static_cast<uint32_t>(kKeyCap);
          if (fits && cl) {
            uint32_t pos = base + inc - cl;
            uint64_t mk = pm;
            while (mk) {
              const int bi = __ffsll(static_cast<long long>(mk)) - 1;
              mk &= mk - 1ull;
              const int col = (tid + (bi / EPV) * kThreads) * EPV + (bi % EPV);
              const float x = Tr::load_s(stage_p, col);
              const float ye = (P.mode == kModeProcessed && c.teff != 1.0f) ? __fdiv_rn(x, c.teff) : x;
              S.keys[pos++] = make_key(ye, vb + static_cast<uint32_t>(tok_of(P, tbase + col)));
            }
          }
          csync();
          SEL_ADD(tid == 0, 2, t_scan);
          SEL_T(t_slow);
          if (!fits) {
            // the reservations do not fit: every warp takes its own back, then
            // the survivors go in vector by vector, the list cut back to kk
            // whenever the next round might not fit (each round re-tests
            // against the raised bound)
            if (lane == 31 && wtot) atomicSub(&S.v->cnt, wtot);
            for (int j = 0; j < sel::kSelVecs; ++j) {
              csync();
              const bool full = static_cast<int>(S.v->cnt) > kKeyCap - kThreads * EPV;
              csync();
              if (full) shrink_row();
              const float thr_j = fmaxf(thr_y, floor_y);
              const uint64_t thr_k = S.v->thr_key;
              const int v = tid + j * kThreads;
              uint64_t kv[EPV];
              uint32_t mask = 0;
#pragma unroll
              for (int e = 0; e < EPV; ++e) kv[e] = 0ull;
              if (((pm >> (j * EPV)) & ((1ull << EPV) - 1ull)) != 0ull && v < nvec) {
                float x[EPV];
                Tr::unpack(sv[v], x);
#pragma unroll
                for (int e = 0; e < EPV; ++e) {
                  if (((pm >> (j * EPV + e)) & 1ull) && x[e] * yscale >= thr_j) {
                    const float ye = (P.mode == kModeProcessed && c.teff != 1.0f) ? __fdiv_rn(x[e], c.teff) : x[e];
                    kv[e] = make_key(ye, vb + static_cast<uint32_t>(tok_of(P, tbase + v * EPV + e)));
                    if (kv[e] >= thr_k) mask |= 1u << e;
                  }
                }
              }
              warp_append_n<EPV>(mask, kv, S.keys, &S.v->cnt, kKeyCap, &S.v->overflow);
            }
            csync();
          }
          SEL_ADD(tid == 0 && !fits, 4, t_slow);
          // keep room for the next stage's survivors; and take the request
          // bound as it stands now (one value for every selector): once there
          // is one, the rest of the row runs without barriers
          if (tid == 0) {
            const uint64_t tnow = ld_relaxed_u64(P.tau + c.r);
            if (tnow > S.v->tau_pref) S.v->tau_pref = tnow;
          }
          const bool crowded = static_cast<int>(S.v->cnt) > kKeyCap - 1024;
          csync();
          fast = S.v->tau_pref != 0ull;
          if (crowded) shrink_row();
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&S.empty[cstage]);
      if (++cstage == P.stages) {
        cstage = 0;
        cphase ^= 1u;
      }
    }
    // ---- row end.  A row whose survivors and table columns fit its slot goes
    // to the finisher warp (the selectors take the next row at once); the
    // others end here: the normaliser from the streamers' partials and the
    // table, then the candidates
    SEL_T(t_end);
    if (tid == 0) W.sel_abort[q] = S.v->abort;
    csync();
    if (W.sel_abort[q]) break;
    const int row_keys = static_cast<int>(sl->kcnt) + ((cand && c.excl) ? pen_n : 0);
    if ((in_slot || !cand) && !sl->kovf && !S.v->overflow && row_keys <= min(P.k2, sel::kSlotKeys)) {
      if (tid == 0) {
        sl->end_by = sel::kEndFinisher;
        mbar_arrive(&W.handoff[q]);   // release: the slot's keys
      }
      continue;
    }
    SEL_CNT(tid == 0, 13, 1);
    if (in_slot) {
      // the slot's written keys join the selectors' list (beside the survivors
      // that did not fit the slot; a full list: the row is read again)
      const int n = min(static_cast<int>(sl->kcnt), sl->kfail);
      const int b0 = static_cast<int>(S.v->cnt);
      if (b0 + n <= kKeyCap) {
        for (int i = tid; i < n; i += kThreads) S.keys[b0 + i] = sl->keys[i];
      }
      csync();
      if (tid == 0) {
        if (b0 + n <= kKeyCap) S.v->cnt = static_cast<uint32_t>(b0 + n);
        else S.v->overflow = 1;
      }
      csync();
    }
    ok = mbar_wait_bounded(&W.rowdone[q], par, &S.v->abort);   // the streamers' partials
    if (!ok) {
      if (!S.v->abort) atomicOr(P.err, GR_DEVERR_TIMEOUT);
      S.v->abort = 1;
    }
    // one decision before the partials are read: a thread whose wait gave up
    // could otherwise take the exact normaliser's collective path alone
    csync();
    if (tid == 0) W.sel_abort[q] = S.v->abort ? 1 : 0;
    csync();
    if (W.sel_abort[q]) break;
    static_assert(sel::kStrWarps <= 32, "one partial per lane");
    float pm_ = (lane < sel::kStrWarps) ? sl->part_m[lane] : -kInf;
    float ps_ = (lane < sel::kStrWarps) ? sl->part_s[lane] : 0.0f;
    // the penalised columns' processed values join the sum (lanes take table entries in turn)
    for (int e = lane; e < pen_n; e += 32) {
      const float y = sl->tab_y[e];
      if (y > pm_) {
        ps_ = (pm_ == -kInf) ? 0.0f : ps_ * fast_exp2((pm_ - y) * kLog2e);
        pm_ = y;
      }
      if (pm_ > -kInf) ps_ += fast_exp2((y - pm_) * kLog2e);
    }
    float M = pm_;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) M = fmaxf(M, __shfl_xor_sync(0xFFFFFFFFu, M, o));
    float tot = (M > -kInf && pm_ > -kInf) ? ps_ * fast_exp2((pm_ - M) * kLog2e) : 0.0f;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) tot += __shfl_xor_sync(0xFFFFFFFFu, tot, o);
    float lse = M + logf(tot);
    if (M > -kInf && !(tot <= 3.0e38f)) {
      // a non-finite streamed sum: the exact two-pass normaliser from global memory
      lse = sel_exact_row_lse<TL>(P, c, st, sl);
    }
    if (tid == 0) {
      W.sel_abort[q] = S.v->abort;
      if (P.lse_out) P.lse_out[c.row] = lse;
    }
    csync();
    if (W.sel_abort[q]) break;
    if (cand) {
      // the penalised columns are candidates with their processed values
      if (c.excl) {
        for (int jb = 0; jb < pen_n; jb += kThreads) {
          const int j = jb + tid;
          bool pred = false;
          uint64_t key = 0ull;
          if (j < pen_n) {
            key = make_key(sl->tab_y[j], vb + static_cast<uint32_t>(tok_of(P, sl->tab_tok[j])));
            pred = key >= S.v->thr_key;
          }
          warp_append(pred, key, S.keys, &S.v->cnt, kKeyCap, &S.v->overflow);
        }
        csync();
      }
      if (S.v->overflow) {
        // the row's survivors did not fit its list: its exact top-2B straight
        // from the row in global memory, and its EOS completion score
        st.rescan_row(c, lse, P.k2, false);
        const int eos_l = (P.eos >= 0) ? col_of(P, P.eos) : -1;
        if (tid == 0 && eos_l >= 0 && P.eos_score)
          P.eos_score[c.row] = __fadd_rn(c.cum, __fsub_rn(st.exact_y(c, st.load_logit(c, eos_l), eos_l), lse));
      } else {
        st.unconstrained_candidates(c, lse);
      }
      if (tid == 0) S.v->thr_key = 0ull;   // only the request bound applies from here
      csync();
      st.emit(c, /*refilter=*/true);
    }
    csync();   // every selector is done with the slot
    SEL_ADD(tid == 0, 5, t_end);
    if (tid == 0) {
      sl->end_by = sel::kEndSelectors;
      mbar_arrive(&W.handoff[q]);
    }
  }
  SEL_ADD(tid == 0, 12, t_sel);
}

// Exact log-sum-exp of a row from global memory by one warp (two passes), the
// penalised columns with their table values: the finisher's rows whose
// streamed sum was not finite.
template <typename TL>
__device__ float sel_exact_row_lse_warp(const Params& P, const RowCtx& c, const sel::Slot* sl, const TL* rowp) {
  const int lane = lane_id();
  const float ys = (P.mode == kModeProcessed) ? c.rteff : 1.0f;
  const int pen_n = sl->pen_n;
  auto yval = [&](int i) -> float {
    const int j = (pen_n > 0) ? sel::table_find(sl, i) : -1;
    return (j >= 0) ? sl->tab_y[j] : LogitTraits<TL>::load1(rowp + i) * ys;
  };
  float M = -kInf;
  for (int i = lane; i < P.VL; i += 32) M = fmaxf(M, yval(i));
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) M = fmaxf(M, __shfl_xor_sync(0xFFFFFFFFu, M, o));
  float tot = 0.0f;
  if (M > -kInf)
    for (int i = lane; i < P.VL; i += 32) tot += fast_exp2((yval(i) - M) * kLog2e);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) tot += __shfl_xor_sync(0xFFFFFFFFu, tot, o);
  return (M == -kInf) ? -kInf : M + logf(tot);
}

// One handed-over row, by the finisher warp: the normaliser (the selectors'
// arithmetic), the EOS completion score, the slot's keys and the table
// columns as score keys, those at or above the request's bound emitted with
// one reservation, and the request histogram raised as emit() does.
template <typename TL>
__device__ bool sel_finish_row(const Params& P, sel::Slot* sl, uint64_t* rowdone, uint32_t par) {
  using Tr = LogitTraits<TL>;
  constexpr int ES = sizeof(TL);
  const Smem S = smem_view(P);
  const int lane = lane_id();
  const int* rec = sl->rec;
  RowCtx c;
  c.row = rec[kMRow];
  c.r = rec[kMR];
  c.b = rec[kMB];
  fill_row_ctx<TL>(P, rec, c);
  const int pen_n = sl->pen_n;
  const TL* rowp = reinterpret_cast<const TL*>(static_cast<const char*>(P.logits) +
                                               static_cast<size_t>(c.row) * static_cast<size_t>(P.row_stride) * ES);
  // the EOS column's logit, fetched while the streamers finish the row
  const int eos_l = (c.stream && P.eos >= 0 && P.eos_score != nullptr) ? col_of(P, P.eos) : -1;
  const float x_eos = (lane == 0 && eos_l >= 0) ? Tr::load1(rowp + eos_l) : 0.0f;
  if (!__all_sync(0xFFFFFFFFu, mbar_wait_bounded(rowdone, par, &S.v->abort))) return false;
  float pm_ = (lane < sel::kStrWarps) ? sl->part_m[lane] : -kInf;
  float ps_ = (lane < sel::kStrWarps) ? sl->part_s[lane] : 0.0f;
  for (int e = lane; e < pen_n; e += 32) {
    const float y = sl->tab_y[e];
    if (y > pm_) {
      ps_ = (pm_ == -kInf) ? 0.0f : ps_ * fast_exp2((pm_ - y) * kLog2e);
      pm_ = y;
    }
    if (pm_ > -kInf) ps_ += fast_exp2((y - pm_) * kLog2e);
  }
  float M = pm_;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) M = fmaxf(M, __shfl_xor_sync(0xFFFFFFFFu, M, o));
  float tot = (M > -kInf && pm_ > -kInf) ? ps_ * fast_exp2((pm_ - M) * kLog2e) : 0.0f;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) tot += __shfl_xor_sync(0xFFFFFFFFu, tot, o);
  float lse = M + logf(tot);
  if (M > -kInf && !(tot <= 3.0e38f)) lse = sel_exact_row_lse_warp<TL>(P, c, sl, rowp);
  if (lane == 0 && P.lse_out) P.lse_out[c.row] = lse;
  if (!c.stream) return true;
  if (lane == 0 && eos_l >= 0) {
    float y = x_eos;
    if (P.mode == kModeProcessed) {
      const int j = c.excl ? sel::table_find(sl, eos_l) : -1;
      y = (j >= 0) ? sl->tab_y[j] : ((c.teff == 1.0f) ? x_eos : __fdiv_rn(x_eos, c.teff));
    }
    P.eos_score[c.row] = __fadd_rn(c.cum, __fsub_rn(y, lse));
  }
  const uint32_t vb = static_cast<uint32_t>(c.b) * static_cast<uint32_t>(P.V);
  const int nk = min(static_cast<int>(sl->kcnt), sel::kSlotKeys);
  const int ntot = nk + (c.excl ? pen_n : 0);
  const uint64_t tau_rec = static_cast<uint64_t>(static_cast<uint32_t>(rec[kMTauLo])) |
                           (static_cast<uint64_t>(static_cast<uint32_t>(rec[kMTauHi])) << 32);
  const uint64_t t_now = ld_relaxed_u64(P.tau + c.r);
  const uint64_t thr = (t_now > tau_rec) ? t_now : tau_rec;   // any value the bound took is a valid one
  auto score_key = [&](int i) -> uint64_t {
    const uint64_t k = (i < nk) ? sl->keys[i]
                                : make_key(sl->tab_y[i - nk], vb + static_cast<uint32_t>(tok_of(P, sl->tab_tok[i - nk])));
    const uint32_t flat = key_flat(k);
    float sc = __fadd_rn(c.cum, __fsub_rn(key_score(k), lse));
    if (static_cast<int>(flat - vb) == P.eos) sc = -kInf;
    return make_key(sc, flat);
  };
  int n_emit = 0;
  for (int i0 = 0; i0 < ntot; i0 += 32) {
    const int i = i0 + lane;
    n_emit += __popc(__ballot_sync(0xFFFFFFFFu, i < ntot && score_key(i) >= thr));
  }
  if (n_emit == 0) return true;
  uint32_t base = 0;
  if (lane == 0) base = atomicAdd(P.rowcnt + static_cast<size_t>(c.r) * P.NB, static_cast<unsigned>(n_emit));
  base = __shfl_sync(0xFFFFFFFFu, base, 0);
  unsigned long long* dst = P.buf + static_cast<size_t>(c.r) * P.NB * static_cast<size_t>(P.k2) + base;
  const uint64_t keep = l2_policy_evict_last();
  unsigned int* gh = P.req_hist ? P.req_hist + static_cast<size_t>(c.r) * kReqHistBins : nullptr;
  const float ref = __int_as_float(rec[kMRef]);
  int pos = 0;
  for (int i0 = 0; i0 < ntot; i0 += 32) {
    const int i = i0 + lane;
    uint64_t k = 0ull;
    bool pass = false;
    if (i < ntot) {
      k = score_key(i);
      pass = k >= thr;
    }
    const unsigned ball = __ballot_sync(0xFFFFFFFFu, pass);
    if (pass) {
      st_keep_u64(dst + pos + __popc(ball & ((1u << lane) - 1u)), k, keep);
      if (gh != nullptr) {
        // the request histogram's bin of this score (as raise_tau_from_histogram)
        const float d = (ref - key_score(k)) * kReqHistScale;
        const int bin = (d < 0.0f) ? 0 : ((d >= 0.0f && d < kReqHistBins - 1) ? static_cast<int>(d) : kReqHistBins - 1);
        atomicAdd(gh + bin, 1u);
      }
    }
    pos += __popc(ball);
  }
  if (gh != nullptr) {
    // the first bin where the count from the top reaches 2B bounds the
    // request's 2B-th key (counts only grow: any snapshot is a lower bound)
    __syncwarp();
    constexpr int kPerLane = kReqHistBins / 32;
    uint32_t mine = 0;
#pragma unroll
    for (int j = 0; j < kPerLane; ++j) {
      const int bin = lane * kPerLane + j;
      if (bin != kReqHistBins - 1) mine += __ldcg(gh + bin);
    }
    uint32_t inc = mine;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const uint32_t v = __shfl_up_sync(0xFFFFFFFFu, inc, o);
      if (lane >= o) inc += v;
    }
    const uint32_t before = inc - mine;
    const uint32_t k2 = static_cast<uint32_t>(P.k2);
    if (before < k2 && before + mine >= k2) {
      uint32_t acc = before;
      for (int j = 0; j < kPerLane; ++j) {
        const int bin = lane * kPerLane + j;
        if (bin == kReqHistBins - 1) break;
        acc += __ldcg(gh + bin);
        if (acc >= k2) {
          const float edge = ref - static_cast<float>(bin + 2) / kReqHistScale;
          const uint64_t cand = static_cast<uint64_t>(f32_to_ord(__fadd_rn(edge, 0.0f))) << 32;
          atomicMax(P.tau + c.r, static_cast<unsigned long long>(cand));
          break;
        }
      }
    }
  }
  return true;
}

// Finisher warp: for every row, once the selectors are done with it, its end
// when they handed it over; then the slot goes back to the producer.
template <typename TL>
__device__ void sel_finish_rows(const Params& P) {
  const Smem S = smem_view(P);
  const sel::View W = sel::view();
  const int lane = lane_id();
  for (int it = 0;; ++it) {
    const int q = it % sel::kSlots;
    const uint32_t par = static_cast<uint32_t>(it / sel::kSlots) & 1u;
    sel::Slot* sl = W.slot(q);
    bool ok = __all_sync(0xFFFFFFFFu, mbar_wait_bounded(&W.recfull[q], par, &S.v->abort));
    if (ok && sl->rec[kMRow] < 0) break;   // no more rows
    if (ok) ok = __all_sync(0xFFFFFFFFu, mbar_wait_bounded(&W.handoff[q], par, &S.v->abort));
    SEL_T(t_fin);
    if (ok && sl->end_by == sel::kEndFinisher) ok = sel_finish_row<TL>(P, sl, &W.rowdone[q], par);
    SEL_ADD(lane == 0, 6, t_fin);
    if (!ok) {
      if (lane == 0) {
        if (!S.v->abort) atomicOr(P.err, GR_DEVERR_TIMEOUT);
        S.v->abort = 1;
      }
      break;
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&W.findone[q]);
  }
}

template <typename TL>
__global__ void __launch_bounds__(sel::kBlockSel, 1) fused_select_ws_kernel(const __grid_constant__ Params P) {
  const Smem S = smem_view(P);
  const sel::View W = sel::view();
  const int tid = threadIdx.x, warp = warp_id();
  if (tid == 0) {
    for (int s = 0; s < P.stages; ++s) {
      mbar_init(&S.full[s], 1);
      mbar_init(&S.empty[s], sel::kStrWarps + sel::kSelWarps);
    }
    for (int q = 0; q < sel::kSlots; ++q) {
      mbar_init(&W.recfull[q], 1);
      mbar_init(&W.rowdone[q], sel::kStrWarps);
      mbar_init(&W.findone[q], 1);
      mbar_init(&W.handoff[q], 1);
    }
    fence_mbar_init();
    S.v->abort = 0;
    S.v->producer_done = 0;
    S.v->issued = 0;
  }
  GR_PROF_INIT();
  pdl_wait();        // row metadata and the zeroed bounds come from the previous kernel
  pdl_trigger();
  __syncthreads();
  if (warp == sel::kFinWarp) {
    sel_finish_rows<TL>(P);
  } else if (warp == sel::kProdWarp) {
    sel_produce<TL>(P);
  } else if (warp >= sel::kSelWarps) {
    sel_stream_rows<TL>(P);
  } else {
    sel_select_rows<TL>(P);
  }
#ifdef GR_PHASE_PROFILE
  __syncthreads();
  GR_PROF_FLUSH();
#endif
}
