// Warp-specialised step kernel: one CTA per SM, three warp roles.
//
//   warps 0..7    finishers  the row end, one row behind the streamers: the
//                            normaliser from the streamers' partials, candidate
//                            scoring against the child window, row slot
//                            emission (the Step helpers, named barrier 1 over
//                            these 256 threads)
//   next warps    streamers  the full-vocabulary (max, sum exp) of each row from
//                            the bulk-copy ring; no barrier among them
//   last warp     producer   row scheduling: the row's metadata record and its
//                            child window (one bulk copy into the row slot's
//                            window), then the row body into the ring
//
// Rows alternate between two slots (record, window, partials).  mbarriers carry
// every hand-off: recfull / winfull (producer -> streamers / finishers),
// rowdone (streamers -> finishers), findone (finishers -> producer: the slot is
// free again), and the ring's full / empty pair.  The streamers only stream,
// so the ring drains at the HBM rate while the finishers work.
//
// Used for steps whose rows need no per-row streamed selection
// (per_beam_k == 0) and no penalty exclusion (not processed mode with penalty
// tensors); a row without a catalog node in such a step is read again by the
// finishers.  Included from gr_beam_step.cu.
#pragma once

#ifndef GR_WS_STREAM_WARPS
#define GR_WS_STREAM_WARPS 16
#endif

namespace ws {
constexpr int kFinWarps = kWarps;                 // finishers are the Step helpers' kThreads
constexpr int kStrWarps = GR_WS_STREAM_WARPS;
constexpr int kStrThreads = kStrWarps * 32;
constexpr int kProdWarp = kFinWarps + kStrWarps;
constexpr int kBlockWs = (kProdWarp + 1) * 32;
#ifndef GR_WS_VPT
#define GR_WS_VPT 4
#endif
constexpr int kVecPerThread = GR_WS_VPT;
constexpr int kStage = kStrThreads * kVecPerThread * 16;   // 4 vectors per streaming thread per stage
constexpr int kMaxStagesWs = kMaxStages;          // full/empty barriers live in the common layout

// Rows rotate through kSlots slots (record, child window, partials), so the
// producer can run two rows ahead of the row-end warps.
#ifndef GR_WS_SLOTS
#define GR_WS_SLOTS 3
#endif
constexpr int kSlots = GR_WS_SLOTS;

// Pieces after the common fixed layout (the penalty pieces are never used here).
constexpr size_t kOffWin1 = kOffWin + align128(size_t(kWinBytes));       // slots 1.. child windows
constexpr size_t kOffRec = kOffWin1 + (kSlots - 1) * align128(size_t(kWinBytes));   // records [kSlots][kMetaWords]
constexpr size_t kOffPart = kOffRec + align128(kSlots * kMetaWords * 4);  // partial m, s [2][kSlots][kStrWarps]
constexpr size_t kOffRowBars = kOffPart + align128(2 * kSlots * kStrWarps * 4);
constexpr size_t kOffFlags = kOffRowBars + align128(4 * kSlots * 8);
constexpr size_t kOffRing = kOffFlags + 128;

__host__ __device__ constexpr size_t smem_bytes(int stages) { return kOffRing + size_t(stages) * kStage; }

// Window byte offset of a slot relative to the common window (slot 0).
__host__ __device__ constexpr int win_off(int slot) {
  return slot ? static_cast<int>(kOffWin1 - kOffWin) + (slot - 1) * static_cast<int>(align128(size_t(kWinBytes))) : 0;
}

struct View {
  int* rec0;           // records [kSlots][kMetaWords]
  float* part_m0;      // partial maxima [kSlots][kStrWarps]
  float* part_s0;      // partial sums [kSlots][kStrWarps]
  uint64_t* recfull;   // [kSlots] producer -> streamers and finishers: record and window bounds written
  uint64_t* winfull;   // [kSlots] producer (bulk copy) -> finishers: window landed
  uint64_t* rowdone;   // [kSlots] streamers -> finishers (one arrival per streaming warp)
  uint64_t* findone;   // [kSlots] finishers -> producer: slot free
  volatile int* fin_abort;   // [kSlots] finishers' per-row abort decision
  int* win_lo;         // [kSlots] first local column of the slot's window
  int* win_hi;         // [kSlots] last local column of the slot's window (win_lo > win_hi: none)
  unsigned char* ring;
  __device__ __forceinline__ int* rec(int slot) const { return rec0 + slot * kMetaWords; }
  __device__ __forceinline__ float* part_m(int slot) const { return part_m0 + slot * kStrWarps; }
  __device__ __forceinline__ float* part_s(int slot) const { return part_s0 + slot * kStrWarps; }
  __device__ __forceinline__ unsigned char* win(int slot) const { return g_smem + kOffWin + win_off(slot); }
};

__device__ __forceinline__ View view() {
  View W;
  W.rec0 = reinterpret_cast<int*>(g_smem + kOffRec);
  W.part_m0 = reinterpret_cast<float*>(g_smem + kOffPart);
  W.part_s0 = W.part_m0 + kSlots * kStrWarps;
  W.recfull = reinterpret_cast<uint64_t*>(g_smem + kOffRowBars);
  W.winfull = W.recfull + kSlots;
  W.rowdone = W.recfull + 2 * kSlots;
  W.findone = W.recfull + 3 * kSlots;
  W.fin_abort = reinterpret_cast<volatile int*>(g_smem + kOffFlags);
  W.win_lo = reinterpret_cast<int*>(g_smem + kOffFlags) + kSlots;
  W.win_hi = W.win_lo + kSlots;
  W.ring = g_smem + kOffRing;
  return W;
}
}  // namespace ws

#ifdef GR_PHASE_PROFILE
#define WS_PROF_T(var) const long long var = clock64()
#define WS_PROF_ADD(cond, slot, t0) \
  do { if (cond) S.v->prof[slot] += clock64() - (t0); } while (0)
#else
#define WS_PROF_T(var)
#define WS_PROF_ADD(cond, slot, t0) do { } while (0)
#endif

// Producer warp: per row, the record and window of its slot, then the body.
// Rows are taken dynamically: each CTA's producer draws the next sequence
// number from a global counter (one row ahead), so CTAs with cheap rows take
// more of them.  A record with row -1 tells the other roles to stop.
template <typename TL>
__device__ void ws_produce(const Params& P) {
  constexpr int ES = sizeof(TL);
  const Smem S = smem_view(P);
  const ws::View W = ws::view();
  const int lane = lane_id();
  const uint64_t pol = l2_policy_evict_first();
  int stage = 0;
  uint32_t round = 0;
  long long fills = 0;
  static_assert(kMetaWords == 32, "one record word per producer lane");
  // the next row's record word (lane = word) and its request threshold (lane 0),
  // loaded one row ahead
  const int total = P.R * P.NB;
  auto draw = [&]() -> int {
    int seq = 0;
    if (lane == 0) seq = static_cast<int>(atomicAdd(P.row_counter, 1u));
    seq = __shfl_sync(0xFFFFFFFFu, seq, 0);
    return (seq < total) ? row_of_seq(P, seq) : -1;
  };
  int meta_word = 0;
  unsigned long long tau_word = 0;
  int row_next = draw();
  if (row_next >= 0) {
    meta_word = __ldcg(P.meta + static_cast<size_t>(row_next) * kMetaWords + lane);
    if (lane == 0) tau_word = *reinterpret_cast<volatile unsigned long long*>(P.tau + row_next / P.NB);
  }
  for (int it = 0;; ++it) {
    const int slot = it % ws::kSlots;
    const int row = row_next;
    // the slot is free once the finishers are done with row it - kSlots
    if (it >= ws::kSlots) {
      WS_PROF_T(t_fd);
      int good = 1;
      if (lane == 0)
        good = mbar_wait_bounded(&W.findone[slot], static_cast<uint32_t>(it / ws::kSlots - 1) & 1u, &S.v->abort) ? 1 : 0;
      WS_PROF_ADD(lane == 0, 6, t_fd);
      if (!__shfl_sync(0xFFFFFFFFu, good, 0)) {
        if (lane == 0) {
          if (!S.v->abort) atomicOr(P.err, GR_DEVERR_TIMEOUT);
          S.v->abort = 1;
        }
        break;
      }
    }
    if (row < 0) {
      // no rows left: a stop record for the streaming and row-end warps
      if (lane == 0) {
        W.rec(slot)[kMRow] = -1;
        mbar_arrive(&W.recfull[slot]);
      }
      break;
    }
    const int cur = meta_word;
    const unsigned long long tau_cur = __shfl_sync(0xFFFFFFFFu, tau_word, 0);
    W.rec(slot)[lane] = (lane == kMTauLo) ? static_cast<int>(tau_cur & 0xFFFFFFFFull)
                      : (lane == kMTauHi) ? static_cast<int>(tau_cur >> 32) : cur;
    row_next = draw();
    if (row_next >= 0) {
      meta_word = __ldcg(P.meta + static_cast<size_t>(row_next) * kMetaWords + lane);
      if (lane == 0) tau_word = *reinterpret_cast<volatile unsigned long long*>(P.tau + row_next / P.NB);
    }
    const int node = __shfl_sync(0xFFFFFFFFu, cur, kMNode);
    const int c0 = __shfl_sync(0xFFFFFFFFu, cur, kMC0);
    const int c1 = __shfl_sync(0xFFFFFFFFu, cur, kMC1);
    const int lt = __shfl_sync(0xFFFFFFFFu, cur, kMLo);
    const int ht = __shfl_sync(0xFFFFFFFFu, cur, kMHi);
    int ok = 1;
    if (lane == 0) {
      // child window: the 16-byte aligned part of the row body that covers the
      // children's column range [lo, hi] (its first kWinBytes); children outside
      // it are read from global memory by the finishers
      const uintptr_t a = reinterpret_cast<uintptr_t>(P.logits) +
                          static_cast<uintptr_t>(row) * static_cast<uintptr_t>(P.row_stride) * ES;
      int wlo = 1, whi = 0;
      uint32_t wbytes = 0;
      if (P.K == 0 && !P.partial_only && !P.stall_copies && node >= 0 && c1 > c0) {
        const int lo = col_ceil(P, lt), hi = min(col_floor(P, ht), P.VL - 1);
        if (lo <= hi) {
          const uintptr_t body0 = (a + 15) & ~uintptr_t(15);
          const uintptr_t body1 = (a + static_cast<uintptr_t>(P.VL) * ES) & ~uintptr_t(15);
          uintptr_t a0 = (a + static_cast<uintptr_t>(lo) * ES) & ~uintptr_t(15);
          if (a0 < body0) a0 = body0;
          uintptr_t a1 = (a + static_cast<uintptr_t>(hi + 1) * ES + 15) & ~uintptr_t(15);
          if (a1 > body1) a1 = body1;
          if (a1 > a0 + kWinBytes) a1 = a0 + kWinBytes;
          if (a1 > a0) {
            wbytes = static_cast<uint32_t>(a1 - a0);
            wlo = static_cast<int>((a0 - a) / ES);
            whi = static_cast<int>((a1 - a) / ES) - 1;
            fence_proxy_async_smem();
            mbar_arrive_expect_tx(&W.winfull[slot], wbytes);
            bulk_copy_g2s_keep(W.win(slot), reinterpret_cast<const void*>(a0), wbytes, &W.winfull[slot]);
          }
        }
      }
      if (wbytes == 0) mbar_arrive(&W.winfull[slot]);
      W.win_lo[slot] = wlo;
      W.win_hi[slot] = whi;
    }
    __syncwarp();
    if (lane == 0) {
      mbar_arrive(&W.recfull[slot]);   // release: the record (every lane's word) and the window bounds
      const Geom g = row_geom<ES, ws::kStage>(P, row);
      // a given normaliser needs no stream (the test hook issues none either)
      const int nchunks = (P.lse_in || P.stall_copies) ? 0 : g.nchunks;
      for (int ch = 0; ch < nchunks; ++ch) {
        if (fills >= P.stages &&
            !mbar_wait_bounded(&S.empty[stage], (round - 1u) & 1u, &S.v->abort)) {
          if (!S.v->abort) atomicOr(P.err, GR_DEVERR_TIMEOUT);
          S.v->abort = 1;
          ok = 0;
          break;
        }
        const long long off = static_cast<long long>(ch) * ws::kStage;
        const uint32_t bytes =
            static_cast<uint32_t>(min(static_cast<long long>(ws::kStage), g.body_bytes - off));
        fence_proxy_async_smem();
        mbar_arrive_expect_tx(&S.full[stage], bytes);
        bulk_copy_g2s(W.ring + static_cast<size_t>(stage) * ws::kStage, g.body + off, bytes, &S.full[stage], pol);
        ++fills;
        if (++stage == P.stages) {
          stage = 0;
          ++round;
        }
      }
    }
    if (!__shfl_sync(0xFFFFFFFFu, ok, 0)) break;
  }
  if (lane == 0) {
    S.v->issued = fills;
    __threadfence_block();
    S.v->producer_done = 1;
  }
}

// Streamers: (max, sum exp) of every row.  Each thread's running reference is
// the first element it sees; the sum is accumulated without overflow checks
// (a non-finite total makes the finishers recompute the row exactly).
template <typename TL>
__device__ void ws_stream_rows(const Params& P) {
  const Smem S = smem_view(P);
  const ws::View W = ws::view();
  using Tr = LogitTraits<TL>;
  constexpr int ES = sizeof(TL);
  constexpr int kVPT = ws::kVecPerThread;
  const int sid = static_cast<int>(threadIdx.x) - ws::kFinWarps * 32;   // 0 .. kStrThreads-1
  const int swarp = sid >> 5, lane = lane_id();
  int cstage = 0;
  uint32_t cphase = 0;
  long long consumed = 0;
  bool aborted = false;
  WS_PROF_T(t_all);
  int rows_done = 0;
  for (int it = 0;; ++it) {
    const int slot = it % ws::kSlots;
    WS_PROF_T(t_rf);
    if (!mbar_wait_bounded(&W.recfull[slot], static_cast<uint32_t>(it / ws::kSlots) & 1u, &S.v->abort)) {
      if (!S.v->abort) atomicOr(P.err, GR_DEVERR_TIMEOUT);
      S.v->abort = 1;
    }
    WS_PROF_ADD(sid == 0, 5, t_rf);
    if (__any_sync(0xFFFFFFFFu, S.v->abort != 0)) {
      aborted = true;
      break;
    }
    const int row = W.rec(slot)[kMRow];
    if (row < 0) break;   // stop record (the same word for every lane)
    ++rows_done;
    const float yscale = (P.mode == kModeProcessed) ? __int_as_float(W.rec(slot)[kMRteff]) : 1.0f;
    const float a = kLog2e * yscale;
    float m = -kInf, s = 0.0f;
    const Geom g = row_geom<ES, ws::kStage>(P, row);
    const int nchunks = P.lse_in ? 0 : g.nchunks;   // a given normaliser needs no stream
    // head / tail columns outside the 16-byte aligned body (exact online update)
    if (!P.lse_in) {
      const int nh = g.head, nt = P.VL - g.tail_start;
      const TL* rowp = reinterpret_cast<const TL*>(g.rowp);
      for (int i = sid; i < nh + nt; i += ws::kStrThreads) {
        const int tl = (i < nh) ? i : g.tail_start + (i - nh);
        const float y = Tr::load1(rowp + tl) * yscale;
        if (y > m) {
          s = s * fast_exp2((m - y) * kLog2e);
          m = y;
        }
        if (m > -kInf) s += fast_exp2((y - m) * kLog2e);
      }
    }
    uint64_t sacc0 = pack2(0.0f, 0.0f), sacc1 = pack2(0.0f, 0.0f);
    WS_PROF_ADD(sid == 0, 14, t_rf);
    WS_PROF_T(t_stream);
    for (int ch = 0; ch < nchunks; ++ch) {
      WS_PROF_T(t_wait);
      if (!mbar_wait_bounded(&S.full[cstage], cphase, &S.v->abort)) {
        if (!S.v->abort) atomicOr(P.err, GR_DEVERR_TIMEOUT);
        S.v->abort = 1;
      }
      WS_PROF_ADD(sid == 0, 1, t_wait);
      const long long off = static_cast<long long>(ch) * ws::kStage;
      const int nvec = static_cast<int>(min(static_cast<long long>(ws::kStage), g.body_bytes - off) >> 4);
      const uint4* sv = reinterpret_cast<const uint4*>(W.ring + static_cast<size_t>(cstage) * ws::kStage);
      uint4 vv[kVPT];
#pragma unroll
      for (int j = 0; j < kVPT; ++j)
        vv[j] = (sid + j * ws::kStrThreads < nvec) ? sv[sid + j * ws::kStrThreads] : make_uint4(0, 0, 0, 0);
      // the stage is in registers now: hand it back to the producer before the math
      __syncwarp();
      if (lane == 0) mbar_arrive(&S.empty[cstage]);
      if (++cstage == P.stages) {
        cstage = 0;
        cphase ^= 1u;
      }
      ++consumed;
      if (ch == 0 && m == -kInf && sid < nvec) {
        float x[Tr::kPerVec];
        Tr::unpack(vv[0], x);
        m = x[0] * yscale;      // any element of the row works as the reference
      }
      const float cm = -m * kLog2e;
      const uint64_t A2 = pack2(a, a), C2 = pack2(cm, cm);
#pragma unroll
      for (int j = 0; j < kVPT; ++j)
        if (sid + j * ws::kStrThreads < nvec) FastSum<TL>::add(vv[j], A2, C2, sacc0, sacc1);
    }
    WS_PROF_ADD(sid == 0, 0, t_stream);
    WS_PROF_T(t_end);
    fold(sacc0, sacc1, s);
    // warp partial of (m, s): the warp maximum, then every lane's sum rescaled
    // to it once and added up; the finishers combine the kStrWarps partials
    float M = m;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) M = fmaxf(M, __shfl_xor_sync(0xFFFFFFFFu, M, o));
    s = (m == -kInf) ? 0.0f : s * fast_exp2((m - M) * kLog2e);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xFFFFFFFFu, s, o);
    m = M;
    if (lane == 0) {
      W.part_m(slot)[swarp] = m;
      W.part_s(slot)[swarp] = s;
      mbar_arrive(&W.rowdone[slot]);   // release: the warp's partial
    }
    WS_PROF_ADD(sid == 0, 13, t_end);
  }
  WS_PROF_ADD(sid == 0, 11, t_all);
#ifdef GR_PHASE_PROFILE
  if (sid == 0) S.v->prof[10] += rows_done;
#endif
  if (aborted && sid == 0) {
    // wait (bounded) for the producer to stop and for its copies still in flight
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
}

// Exact log-sum-exp of a row from global memory (two passes), for rows whose
// streamed sum was not finite.  Finisher threads only.
template <typename TL>
__device__ float ws_exact_row_lse(const Params& P, const RowCtx& c, const Step<TL>& st) {
  const Smem S = smem_view(P);
  const int tid = threadIdx.x, lane = lane_id(), warp = warp_id();
  const float ys = (P.mode == kModeProcessed) ? c.rteff : 1.0f;
  float mx = -kInf;
  for (int i = tid; i < P.VL; i += kThreads) mx = fmaxf(mx, st.load_logit(c, i) * ys);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xFFFFFFFFu, mx, o));
  if (lane == 0) S.red_m[warp] = mx;
  csync();
  float M = -kInf;
#pragma unroll
  for (int w = 0; w < kWarps; ++w) M = fmaxf(M, S.red_m[w]);
  float sm = 0.0f;
  if (M > -kInf)
    for (int i = tid; i < P.VL; i += kThreads) sm += fast_exp2((st.load_logit(c, i) * ys - M) * kLog2e);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) sm += __shfl_xor_sync(0xFFFFFFFFu, sm, o);
  if (lane == 0) S.red_s[warp] = sm;
  csync();
  float tot = 0.0f;
#pragma unroll
  for (int w = 0; w < kWarps; ++w) tot += S.red_s[w];
  csync();   // red_m / red_s are free again
  return (M == -kInf) ? -kInf : M + logf(tot);
}

// Finishers: row end of every row, one row behind the streamers.
template <typename TL>
__device__ void ws_finish_rows(const Params& P) {
  const Smem S = smem_view(P);
  const ws::View W = ws::view();
  Step<TL> st(P);
  using Tr = LogitTraits<TL>;
  constexpr int EPV = Tr::kPerVec;
  const int tid = threadIdx.x, lane = lane_id(), warp = warp_id();
  for (int it = 0;; ++it) {
    const int slot = it % ws::kSlots;
    const uint32_t par = static_cast<uint32_t>(it / ws::kSlots) & 1u;
    WS_PROF_T(t_rd);
    bool ok = mbar_wait_bounded(&W.recfull[slot], par, &S.v->abort);
    // a stop record has no row behind it (no partials, no window)
    if (!(ok && W.rec(slot)[kMRow] < 0)) {
      ok = ok && mbar_wait_bounded(&W.rowdone[slot], par, &S.v->abort);
      ok = ok && mbar_wait_bounded(&W.winfull[slot], par, &S.v->abort);
    }
    if (!ok) {
      if (!S.v->abort) atomicOr(P.err, GR_DEVERR_TIMEOUT);
      S.v->abort = 1;
    }
    // One decision for every finisher before any reads the row: a wait that
    // gave up on one thread (its abort is visible after the barrier) or the
    // stop record ends the loop for all.  Taken per thread, threads that left
    // would be missing at the next barrier, and threads that read partials
    // not yet written could disagree on the exact normaliser's collective path.
    csync();
    if (tid == 0) W.fin_abort[slot] = (S.v->abort || W.rec(slot)[kMRow] < 0) ? 1 : 0;
    csync();
    if (W.fin_abort[slot]) break;
    WS_PROF_ADD(tid == 0, 2, t_rd);
    WS_PROF_T(t_fin);
    RowCtx c;
    const int* rec = W.rec(slot);
    c.row = rec[kMRow];
    c.r = rec[kMR];
    c.b = rec[kMB];
    // a fresh read of the request's running threshold, used at the end of the prelude
    uint64_t tau_fresh = 0;
    if (tid == 0) tau_fresh = *reinterpret_cast<volatile unsigned long long*>(P.tau + c.r);
    fill_row_ctx<TL>(P, rec, c);
    if (c.constrained) {
      c.wlo = W.win_lo[slot];
      c.whi = W.win_hi[slot];
    }
    st.rec = rec;
    st.win_off = ws::win_off(slot);
    // normaliser: lane w of every finisher warp takes streamer partial w; the
    // same shuffle tree in every warp gives every thread the same value
    static_assert(ws::kStrWarps <= 32, "one partial per lane");
    const float pm = (lane < ws::kStrWarps) ? W.part_m(slot)[lane] : -kInf;
    const float ps = (lane < ws::kStrWarps) ? W.part_s(slot)[lane] : 0.0f;
    float M = pm;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) M = fmaxf(M, __shfl_xor_sync(0xFFFFFFFFu, M, o));
    float tot = (M > -kInf && lane < ws::kStrWarps) ? ps * fast_exp2((pm - M) * kLog2e) : 0.0f;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) tot += __shfl_xor_sync(0xFFFFFFFFu, tot, o);
    float lse = M + logf(tot);
    if (P.lse_in) {
      lse = P.lse_in[c.row];   // vocab-sharded phase 2: the global normaliser
    } else if (M > -kInf && !(tot <= 3.0e38f)) {
      // an overflowing or NaN streamed sum (uniform: every finisher has the same tot)
      lse = ws_exact_row_lse<TL>(P, c, st);
      if (P.partial_only) {
        M = lse;
        tot = 1.0f;
      }
    }
    if (tid == 0) {
      // the request's running threshold as the producer read it (a stale bound is still valid)
      uint64_t tau_pref = static_cast<uint64_t>(static_cast<uint32_t>(rec[kMTauLo])) |
                          (static_cast<uint64_t>(static_cast<uint32_t>(rec[kMTauHi])) << 32);
      if (tau_fresh > tau_pref) tau_pref = tau_fresh;
      S.v->cnt = 0;
      S.v->overflow = 0;
      S.v->discard = 0;
      S.v->tau_pref = tau_pref;
      S.v->thr_key = c.constrained ? tau_pref : 0ull;
      S.v->thr_y = -kInf;
      W.fin_abort[slot] = S.v->abort;
      if (P.partial_only) {
        P.partials[c.row] = make_float2(M, tot);
      } else {
        if (P.lse_out) P.lse_out[c.row] = lse;
        if (P.eos_score) P.eos_score[c.row] = __int_as_float(0x7FC00000);
      }
    }
    csync();
    WS_PROF_ADD(tid == 0, 7, t_fin);
    if (W.fin_abort[slot]) break;
    if (P.partial_only) {
      // vocab-sharded phase 1: the partial is all this row needs
      if (tid == 0) mbar_arrive(&W.findone[slot]);
      continue;
    }
    if (c.constrained) {
      WS_PROF_T(t_cc);
      st.constrained_candidates(c, lse);
      WS_PROF_ADD(tid == 0, 12, t_cc);
    } else if (c.stream) {
      // a row without a catalog node: its selection needs the whole row, which
      // the streamers did not keep, so read it again (L2 or HBM)
      float dm = -kInf, ds = 0.0f, thr_y = -kInf;
      uint64_t thr_key = 0ull;
      const Geom g = row_geom<sizeof(TL)>(P, c.row);
      {
        const int nh = g.head, nt = P.VL - g.tail_start;
        for (int ib = warp * 32; ib < nh + nt; ib += kThreads) {
          const int i = ib + lane;
          const bool valid = i < nh + nt;
          const int tl = valid ? ((i < nh) ? i : g.tail_start + (i - nh)) : 0;
          float x[1];
          x[0] = valid ? st.load_logit(c, tl) : -kInf;
          st.template process<1>(c, x, tl, valid, dm, ds, thr_y, thr_key);
        }
      }
      const uint4* bv = reinterpret_cast<const uint4*>(g.body);
      const int nvec_all = static_cast<int>(g.body_bytes >> 4);
      uint64_t tau_seen = 0ull;
      for (int sb = 0; sb < nvec_all; sb += P.sub_vecs) {
        const int send = min(nvec_all, sb + P.sub_vecs);
        // the request bound as read one sub-batch earlier; this pass knows the
        // row's lse exactly, so the bound needs no estimate of it
        float tau_off = -kInf;
        if (tau_seen) {
          const float ts = key_score(tau_seen);
          const float f = ts - c.cum + lse;
          // margin for the roundings of the exact score (relative to its terms)
          tau_off = f - 1.0e-5f * (fabsf(f) + fabsf(ts) + fabsf(c.cum) + fabsf(lse)) - 1e-30f;
        }
        tau_seen = *reinterpret_cast<volatile unsigned long long*>(P.tau + c.r);
        for (int vb = sb + warp * 32; vb < send; vb += kThreads) {
          const int v = vb + lane;
          const bool valid = v < send;
          float x[EPV];
          if (valid) {
            Tr::unpack(__ldcg(bv + v), x);
          } else {
#pragma unroll
            for (int i = 0; i < EPV; ++i) x[i] = -kInf;
          }
          st.template process<EPV>(c, x, g.head + v * EPV, valid, dm, ds, thr_y, thr_key, tau_off);
        }
        if (st.list_len_sync() > kKeyCap - P.sub_vecs * EPV) {
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
        }
      }
      st.unconstrained_candidates(c, lse);
      if (tid == 0) S.v->thr_key = 0ull;   // only the request bound applies from here
      csync();
    }
    WS_PROF_ADD(tid == 0, 3, t_fin);
    WS_PROF_T(t_emit);
    if (tid == 0 && S.v->overflow) atomicOr(P.err, GR_DEVERR_OVERFLOW);
    st.emit(c, /*refilter=*/!c.constrained);
    csync();   // every finisher is done with the slot's record, window and partials
    if (tid == 0) mbar_arrive(&W.findone[slot]);
    WS_PROF_ADD(tid == 0, 4, t_emit);
  }
}

template <typename TL>
__global__ void __launch_bounds__(ws::kBlockWs, 1) fused_step_ws_kernel(const __grid_constant__ Params P) {
  const Smem S = smem_view(P);
  const ws::View W = ws::view();
  const int tid = threadIdx.x, warp = warp_id();
  if (tid == 0) {
    for (int s = 0; s < P.stages; ++s) {
      mbar_init(&S.full[s], 1);
      mbar_init(&S.empty[s], ws::kStrWarps);
    }
    for (int q = 0; q < ws::kSlots; ++q) {
      mbar_init(&W.recfull[q], 1);
      mbar_init(&W.winfull[q], 1);
      mbar_init(&W.rowdone[q], ws::kStrWarps);
      mbar_init(&W.findone[q], 1);
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
  if (warp == ws::kProdWarp) {
    ws_produce<TL>(P);
  } else if (warp >= ws::kFinWarps) {
    ws_stream_rows<TL>(P);
  } else {
    ws_finish_rows<TL>(P);
  }
#ifdef GR_PHASE_PROFILE
  __syncthreads();
  GR_PROF_FLUSH();
#endif
}
