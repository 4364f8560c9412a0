// gr_device.cuh — device building blocks of the constrained beam step (sm_100a).
//
//  * mbarrier + cp.async.bulk (TMA bulk copy, no tensor map, no multicast)
//    global -> shared staging, with bounded waits that report instead of hang;
//  * order-preserving 64-bit candidate keys: (ord(score) << 32) | ~flat, so
//    that a larger key is a better candidate under the canonical order
//    "score descending, then flat index parent*V+token ascending";
//  * CTA-wide MSB-first radix select (8-bit digits, warp-aggregated shared
//    histograms), in-place compaction and a bitonic sort of keys.
#pragma once

#include <cstdint>
#include <cuda_bf16.h>
#include <cuda_fp16.h>

namespace gr {

constexpr int kThreads = 256;                 // consumer threads per CTA (two CTAs per SM)
constexpr int kBlock = kThreads + 32;         // + one producer warp
constexpr int kWarps = kThreads / 32;
constexpr int kStageBytes = 16384;            // one TMA bulk copy per stage
constexpr int kMaxStages = 8;
constexpr int kWinBytes = 16384;              // child window, raw logits of the row
constexpr int kKeyCap = 4096;                 // candidate keys in shared memory
constexpr int kBatch = 2048;                  // max insertions between capacity checks
constexpr int kPenTableMax = 1024;            // max history tokens with penalties
constexpr int kSlack = 64;                    // extra keys kept by streamed top-k
constexpr int kMaxBitmapWords = 8192;         // penalties: local vocab <= 262144
// Longest time any wait of the step kernels spins before it gives up with
// GR_DEVERR_TIMEOUT (a build may set it lower, e.g. -DGR_WAIT_LIMIT_NS=1000000
// for 1 ms in a test build).
#ifndef GR_WAIT_LIMIT_NS
#define GR_WAIT_LIMIT_NS 2000000000ull
#endif
constexpr unsigned long long kWaitLimitNs = GR_WAIT_LIMIT_NS;   // 2 s per wait by default
constexpr uint32_t kWaitSleepNs = 100000u;                    // longest sleep per try (0.1 ms)

constexpr float kLog2e = 1.4426950408889634f;
#define kInf (__int_as_float(0x7f800000))

// ---------------------------------------------------------------- PTX helpers
// Barrier among the kThreads consumer threads only (named barrier 1); the
// producer warp never takes part, so it can keep prefetching meanwhile.
__device__ __forceinline__ void csync() { asm volatile("bar.sync 1, %0;" ::"n"(kThreads) : "memory"); }

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
               : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}\n"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// As mbar_try_wait, but the thread may sleep (not spin) for up to hint_ns
// nanoseconds; it wakes as soon as the phase completes.
__device__ __forceinline__ bool mbar_try_wait_sleep(uint64_t* bar, uint32_t parity, uint32_t hint_ns) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}\n"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity), "r"(hint_ns)
      : "memory");
  return ok != 0;
}

__device__ __forceinline__ uint64_t global_timer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// Wait for the phase with the given parity to complete.  Gives up (false)
// after kWaitLimitNs, or as soon as *abort is set when abort is non-null.
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t* bar, uint32_t parity,
                                                  const volatile int* abort = nullptr) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = global_timer_ns();
  while (true) {
#ifdef GR_WAIT_SLEEP
    // sleep rather than spin, so that waiting warps leave the issue slots to the others
    if (mbar_try_wait_sleep(bar, parity, kWaitSleepNs)) return true;
#else
    if (mbar_try_wait(bar, parity)) return true;
#endif
    if (abort != nullptr && *abort) return false;
    if (global_timer_ns() - t0 > kWaitLimitNs) return false;
  }
}

__device__ __forceinline__ uint64_t l2_policy_evict_first() {
  uint64_t pol;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(pol));
  return pol;
}

// Bulk copy `bytes` (multiple of 16, both addresses 16-byte aligned) from this
// GPU's global memory into this CTA's shared memory; completion is signalled
// on `bar` as transaction bytes.  No cluster multicast.
__device__ __forceinline__ void bulk_copy_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar,
                                              uint64_t policy) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint"
      " [%0], [%1], %2, [%3], %4;" ::"r"(smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar)), "l"(policy)
      : "memory");
}

// L2 policy that keeps lines resident ahead of streamed (evict-first) data:
// for the small per-step buffers the next kernel reads back.
__device__ __forceinline__ uint64_t l2_policy_evict_last() {
  uint64_t pol;
  asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(pol));
  return pol;
}
// A relaxed GPU-scope 64-bit load: sees other CTAs' atomics, and orders
// nothing around it (a volatile access would keep later loads behind it).
__device__ __forceinline__ unsigned long long ld_relaxed_u64(const unsigned long long* p) {
  unsigned long long v;
  asm volatile("ld.relaxed.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(p));
  return v;
}
__device__ __forceinline__ void st_keep_u64(unsigned long long* p, unsigned long long v, uint64_t pol) {
  asm volatile("st.global.L2::cache_hint.u64 [%0], %1, %2;" ::"l"(p), "l"(v), "l"(pol) : "memory");
}
__device__ __forceinline__ void st_keep_u32(unsigned* p, unsigned v, uint64_t pol) {
  asm volatile("st.global.L2::cache_hint.u32 [%0], %1, %2;" ::"l"(p), "r"(v), "l"(pol) : "memory");
}
__device__ __forceinline__ void st_keep_v4(int4* p, int4 v, uint64_t pol) {
  asm volatile("st.global.L2::cache_hint.v4.s32 [%0], {%1, %2, %3, %4}, %5;" ::"l"(p), "r"(v.x), "r"(v.y), "r"(v.z),
               "r"(v.w), "l"(pol)
               : "memory");
}

// As bulk_copy_g2s with the default L2 policy (the bytes are read again soon).
__device__ __forceinline__ void bulk_copy_g2s_keep(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1], %2, [%3];" ::"r"(smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

__device__ __forceinline__ float fast_exp2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// Packed float2 arithmetic (sm_100: one instruction for two lanes of f32).
__device__ __forceinline__ uint64_t pack2(float lo, float hi) {
  uint64_t r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(lo), "f"(hi));
  return r;
}
__device__ __forceinline__ void unpack2(uint64_t v, float& lo, float& hi) {
  asm("mov.b64 {%0, %1}, %2;" : "=f"(lo), "=f"(hi) : "l"(v));
}
__device__ __forceinline__ uint64_t ffma2(uint64_t a, uint64_t b, uint64_t c) {
  uint64_t d;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
  return d;
}
__device__ __forceinline__ uint64_t fadd2(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}

// 2^t for a pair of floats on the FMA pipe (so that part of a row's
// exponentials leave the MUFU unit): Cody-Waite style range reduction
// t = n + f, n = round(t), |f| <= 1/2, then a degree-5 polynomial for 2^f
// (coefficients fitted here by iteratively reweighted least squares for
// minimax relative error on [-1/2, 1/2]; max relative error 2.4e-7 in float32
// Horner form) and n added to the exponent field.  t is clamped to
// [-125, 128]: results below 2^-125 are negligible next to the sums they enter,
// and t >= 128 yields inf or NaN, as the hardware exp2 overflows.  NaN in gives
// NaN out.
constexpr float kP0 = 1.0000001192092896f, kP1 = 0.6931469440460205f, kP2 = 0.24022120237350464f;
constexpr float kP3 = 0.05550713092088699f, kP4 = 0.009675541892647743f, kP5 = 0.0013276472454890609f;

__device__ __forceinline__ uint64_t poly_exp2x2(uint64_t t2) {
  float t0, t1;
  asm("mov.b64 {%0, %1}, %2;" : "=f"(t0), "=f"(t1) : "l"(t2));
  asm("max.NaN.f32 %0, %0, 0fC2FA0000;" : "+f"(t0));   // -125
  asm("max.NaN.f32 %0, %0, 0fC2FA0000;" : "+f"(t1));
  asm("min.NaN.f32 %0, %0, 0f43000000;" : "+f"(t0));   // 128
  asm("min.NaN.f32 %0, %0, 0f43000000;" : "+f"(t1));
  uint64_t tt;
  asm("mov.b64 %0, {%1, %2};" : "=l"(tt) : "f"(t0), "f"(t1));
  const uint64_t r = fadd2(tt, pack2(12582912.0f, 12582912.0f));   // 1.5 * 2^23: round to integer
  const uint64_t n = fadd2(r, pack2(-12582912.0f, -12582912.0f));
  const uint64_t f = ffma2(n, pack2(-1.0f, -1.0f), tt);              // t - n, exact
  uint64_t p = ffma2(pack2(kP5, kP5), f, pack2(kP4, kP4));
  p = ffma2(p, f, pack2(kP3, kP3));
  p = ffma2(p, f, pack2(kP2, kP2));
  p = ffma2(p, f, pack2(kP1, kP1));
  p = ffma2(p, f, pack2(kP0, kP0));
  float r0, r1, p0, p1;
  unpack2(r, r0, r1);
  unpack2(p, p0, p1);
  // the low bits of r hold n: n << 23 added to the exponent of 2^f
  const float e0 = __uint_as_float(__float_as_uint(r0) * 0x800000u + __float_as_uint(p0));
  const float e1 = __uint_as_float(__float_as_uint(r1) * 0x800000u + __float_as_uint(p1));
  return pack2(e0, e1);
}

// ---------------------------------------------------------------- keys
__device__ __forceinline__ uint32_t f32_to_ord(float f) {
  const uint32_t u = __float_as_uint(f);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

__device__ __forceinline__ float ord_to_f32(uint32_t o) {
  const uint32_t u = (o & 0x80000000u) ? (o & 0x7FFFFFFFu) : ~o;
  return __uint_as_float(u);
}

// Larger key = better candidate: higher score, then lower flat index.
__device__ __forceinline__ uint64_t make_key(float score, uint32_t flat) {
  score = __fadd_rn(score, 0.0f);  // -0 -> +0 so that equal scores tie
  return (static_cast<uint64_t>(f32_to_ord(score)) << 32) | static_cast<uint64_t>(0xFFFFFFFFu - flat);
}

__device__ __forceinline__ float key_score(uint64_t k) { return ord_to_f32(static_cast<uint32_t>(k >> 32)); }
__device__ __forceinline__ uint32_t key_flat(uint64_t k) { return 0xFFFFFFFFu - static_cast<uint32_t>(k); }

// ---------------------------------------------------------------- warp helpers
__device__ __forceinline__ int lane_id() { return threadIdx.x & 31; }
__device__ __forceinline__ int warp_id() { return threadIdx.x >> 5; }

// Append `key` to keys[*cnt] for the lanes with `pred`.  Must be called by all
// 32 lanes of the warp (warp-uniform control flow).
__device__ __forceinline__ void warp_append(bool pred, uint64_t key, uint64_t* keys, uint32_t* cnt,
                                            uint32_t cap, int* overflow) {
  const unsigned bal = __ballot_sync(0xFFFFFFFFu, pred);
  if (bal == 0) return;
  const int lane = lane_id();
  const int leader = __ffs(bal) - 1;
  uint32_t base = 0;
  if (lane == leader) base = atomicAdd(cnt, static_cast<uint32_t>(__popc(bal)));
  base = __shfl_sync(0xFFFFFFFFu, base, leader);
  if (pred) {
    const uint32_t pos = base + __popc(bal & ((1u << lane) - 1u));
    if (pos < cap)
      keys[pos] = key;
    else
      *overflow = 1;
  }
}

// Append the keys kv[i] with bit i of `mask` set (N per lane) with one
// reservation for the whole warp: a warp scan of the lanes' counts gives each
// lane its offset.  Must be called by all 32 lanes of the warp.
template <int N>
__device__ __forceinline__ void warp_append_n(uint32_t mask, const uint64_t (&kv)[N], uint64_t* keys, uint32_t* cnt,
                                              uint32_t cap, int* overflow) {
  const int lane = lane_id();
  const uint32_t c = static_cast<uint32_t>(__popc(mask));
  uint32_t inc = c;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const uint32_t v = __shfl_up_sync(0xFFFFFFFFu, inc, o);
    if (lane >= o) inc += v;
  }
  const uint32_t total = __shfl_sync(0xFFFFFFFFu, inc, 31);
  if (total == 0) return;
  uint32_t base = 0;
  if (lane == 31) base = atomicAdd(cnt, total);
  base = __shfl_sync(0xFFFFFFFFu, base, 31);
  uint32_t pos = base + inc - c;
#pragma unroll
  for (int i = 0; i < N; ++i) {
    if ((mask >> i) & 1u) {
      if (pos < cap)
        keys[pos] = kv[i];
      else
        *overflow = 1;
      ++pos;
    }
  }
}

// Reserve c slots per lane in a shared list with one atomic per warp; returns
// this lane's first slot.  Must be called by all 32 lanes of the warp.
__device__ __forceinline__ uint32_t warp_reserve(uint32_t c, uint32_t* cnt) {
  const int lane = lane_id();
  uint32_t inc = c;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const uint32_t v = __shfl_up_sync(0xFFFFFFFFu, inc, o);
    if (lane >= o) inc += v;
  }
  const uint32_t total = __shfl_sync(0xFFFFFFFFu, inc, 31);
  uint32_t base = 0;
  if (lane == 31 && total > 0) base = atomicAdd(cnt, total);
  base = __shfl_sync(0xFFFFFFFFu, base, 31);
  return base + inc - c;
}

// Programmatic dependent launch: a kernel launched with programmatic stream
// serialization may start before its predecessor in the stream has finished;
// pdl_wait() blocks until the predecessor grid has completed and its memory is
// visible (a no-op for an ordinary launch), pdl_trigger() lets the successor
// grid launch early.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

// ---------------------------------------------------------------- radix select
// Keys kept by a selection: (key >> shift) >= (prefix >> shift).
struct Cut {
  uint64_t prefix;
  int shift;
  __device__ __forceinline__ bool keep(uint64_t k) const { return (k >> shift) >= (prefix >> shift); }
  // A value every kept key is >= to (lower bound of the k-th largest key).
  __device__ __forceinline__ uint64_t floor_key() const {
    return shift >= 64 ? 0ull : (prefix >> shift) << shift;
  }
};

struct SelectScratch {
  uint32_t hist[256];
  uint32_t digit, above, count, pad;
};

// The k largest of n distinct keys (1 <= k <= n), MSB-first over 8-bit digits.
// keyf(i) returns key i.  All threads of the CTA call this.
template <class KeyFn>
__device__ Cut cta_radix_select(KeyFn keyf, int n, int k, SelectScratch* sc, int stop_shift = 0) {
  uint64_t prefix = 0;
  int shift = 64;
  int krem = k;
  const int lane = lane_id();
  while (true) {
    shift -= 8;
    for (int i = threadIdx.x; i < 256; i += kThreads) sc->hist[i] = 0;
    csync();
    const int hs = shift + 8;
    // plain shared-memory atomics (measured faster here than match-based aggregation)
    for (int i = threadIdx.x; i < n; i += kThreads) {
      const uint64_t key = keyf(i);
      if ((hs >= 64) || ((key >> hs) == (prefix >> hs))) atomicAdd(&sc->hist[(key >> shift) & 0xFFu], 1u);
    }
    csync();
    if (warp_id() == 0) {
      uint32_t c[8];
      uint32_t sum = 0;
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        c[j] = sc->hist[255 - 8 * lane - j];
        sum += c[j];
      }
      uint32_t inc = sum;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const uint32_t v = __shfl_up_sync(0xFFFFFFFFu, inc, o);
        if (lane >= o) inc += v;
      }
      const uint32_t exc = inc - sum;
      if (exc < static_cast<uint32_t>(krem) && static_cast<uint32_t>(krem) <= inc) {
        uint32_t acc = exc;
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          if (acc + c[j] >= static_cast<uint32_t>(krem)) {
            sc->digit = 255u - 8u * lane - j;
            sc->above = acc;
            sc->count = c[j];
            break;
          }
          acc += c[j];
        }
      }
    }
    csync();
    const uint32_t d = sc->digit, above = sc->above, cnt = sc->count;
    csync();
    prefix |= static_cast<uint64_t>(d) << shift;
    krem -= static_cast<int>(above);
    // (stop_shift > 0: only the key's bits above stop_shift are resolved)
    if (cnt == static_cast<uint32_t>(krem) || shift <= stop_shift) break;
  }
  return Cut{prefix, shift};
}

// Keep keys[i] (i < n, n <= kKeyCap) with cut.keep(); compacted to the front.
// Returns the new count (also in *cnt).
__device__ __forceinline__ uint32_t cta_compact(uint64_t* keys, int n, Cut cut, uint32_t* cnt) {
  constexpr int kPer = kKeyCap / kThreads;
  uint64_t reg[kPer];
#pragma unroll
  for (int j = 0; j < kPer; ++j) {
    const int i = threadIdx.x + j * kThreads;
    reg[j] = (i < n) ? keys[i] : 0ull;
  }
  csync();
  if (threadIdx.x == 0) *cnt = 0;
  csync();
  int dummy = 0;
  uint32_t mask = 0;
#pragma unroll
  for (int j = 0; j < kPer; ++j) {
    const int i = threadIdx.x + j * kThreads;
    if ((i < n) && cut.keep(reg[j])) mask |= 1u << j;
  }
  warp_append_n<kPer>(mask, reg, keys, cnt, kKeyCap, &dummy);
  csync();
  return *cnt;
}

// Sort a[0..kThreads*E) descending (bitonic).  Thread t holds elements
// [t*E, t*E + E) in registers: exchange distances below E stay in the thread,
// below 32E go through warp shuffles, and only the longer ones through shared
// memory (a[] is the exchange buffer and receives the result).
template <int E>
__device__ __forceinline__ void cta_bitonic_sort_regs_desc(uint64_t* a) {
  constexpr int P = kThreads * E;
  const int tid = threadIdx.x;
  uint64_t v[E];
#pragma unroll
  for (int e = 0; e < E; ++e) v[e] = a[tid * E + e];
  csync();
  for (int k = 2; k <= P; k <<= 1) {
    for (int j = k >> 1; j > 0; j >>= 1) {
      uint64_t o[E];
      if (j < E) {
        // in-thread partners; j is a run-time value, so pick among fixed indices
#pragma unroll
        for (int e = 0; e < E; ++e) o[e] = (j == 1) ? v[e ^ 1] : ((j == 2) ? v[(e ^ 2) % E] : v[(e ^ 4) % E]);
      } else if (j < 32 * E) {
        const int lanes = j / E;
#pragma unroll
        for (int e = 0; e < E; ++e) o[e] = __shfl_xor_sync(0xFFFFFFFFu, v[e], lanes);
      } else {
#pragma unroll
        for (int e = 0; e < E; ++e) a[tid * E + e] = v[e];
        csync();
#pragma unroll
        for (int e = 0; e < E; ++e) o[e] = a[(tid * E + e) ^ j];
        csync();
      }
#pragma unroll
      for (int e = 0; e < E; ++e) {
        const int i = tid * E + e;
        const bool lower = (i & j) == 0;          // i < i ^ j
        const bool desc = (i & k) == 0;           // this run sorts descending
        const bool take_max = (lower == desc);
        v[e] = take_max ? (v[e] > o[e] ? v[e] : o[e]) : (v[e] < o[e] ? v[e] : o[e]);
      }
    }
  }
#pragma unroll
  for (int e = 0; e < E; ++e) a[tid * E + e] = v[e];
  csync();
}

// Sort a[0..P) descending; P a power of two.
__device__ __forceinline__ void cta_bitonic_sort_desc(uint64_t* a, int P) {
  for (int k = 2; k <= P; k <<= 1) {
    for (int j = k >> 1; j > 0; j >>= 1) {
      for (int i = threadIdx.x; i < P; i += kThreads) {
        const int ixj = i ^ j;
        if (ixj > i) {
          const uint64_t x = a[i], y = a[ixj];
          const bool first_half = (i & k) == 0;
          if (first_half ? (x < y) : (x > y)) {
            a[i] = y;
            a[ixj] = x;
          }
        }
      }
      csync();
    }
  }
}

// ---------------------------------------------------------------- logit loads
template <typename TL> struct LogitTraits;
template <> struct LogitTraits<float> {
  static constexpr int kPerVec = 4;
  __device__ static __forceinline__ void unpack(const uint4& v, float* x) {
    x[0] = __uint_as_float(v.x); x[1] = __uint_as_float(v.y);
    x[2] = __uint_as_float(v.z); x[3] = __uint_as_float(v.w);
  }
  __device__ static __forceinline__ float load1(const float* p) { return __ldg(p); }
  // element i of a shared-memory copy
  __device__ static __forceinline__ float load_s(const unsigned char* base, int i) {
    return reinterpret_cast<const float*>(base)[i];
  }
  // set the elements whose bit is set in fl (bit i = element i) to -inf
  __device__ static __forceinline__ void mask_neg_inf(uint4& v, uint32_t fl) {
    if (fl & 1u) v.x = 0xFF800000u;
    if (fl & 2u) v.y = 0xFF800000u;
    if (fl & 4u) v.z = 0xFF800000u;
    if (fl & 8u) v.w = 0xFF800000u;
  }
};

// 2-byte logits: element 2k is the low half of word k, element 2k+1 the high half
__device__ __forceinline__ void mask_neg_inf_u16(uint4& v, uint32_t fl, uint32_t ninf) {
  uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    if ((fl >> (2 * k)) & 1u) w[k] = (w[k] & 0xFFFF0000u) | ninf;
    if ((fl >> (2 * k + 1)) & 1u) w[k] = (w[k] & 0x0000FFFFu) | (ninf << 16);
  }
  v = make_uint4(w[0], w[1], w[2], w[3]);
}
template <> struct LogitTraits<__nv_bfloat16> {
  static constexpr int kPerVec = 8;
  __device__ static __forceinline__ void unpack(const uint4& v, float* x) {
    const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      x[2 * i] = __uint_as_float(w[i] << 16);
      x[2 * i + 1] = __uint_as_float(w[i] & 0xFFFF0000u);
    }
  }
  __device__ static __forceinline__ float load1(const __nv_bfloat16* p) {
    const unsigned short u = __ldg(reinterpret_cast<const unsigned short*>(p));
    return __uint_as_float(static_cast<uint32_t>(u) << 16);
  }
  __device__ static __forceinline__ float load_s(const unsigned char* base, int i) {
    return __uint_as_float(static_cast<uint32_t>(reinterpret_cast<const unsigned short*>(base)[i]) << 16);
  }
  __device__ static __forceinline__ void mask_neg_inf(uint4& v, uint32_t fl) { mask_neg_inf_u16(v, fl, 0xFF80u); }
};
template <> struct LogitTraits<__half> {
  static constexpr int kPerVec = 8;
  __device__ static __forceinline__ void unpack(const uint4& v, float* x) {
    const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      __half2 h = *reinterpret_cast<const __half2*>(&w[i]);
      float2 f = __half22float2(h);
      x[2 * i] = f.x;
      x[2 * i + 1] = f.y;
    }
  }
  __device__ static __forceinline__ float load1(const __half* p) { return __half2float(__ldg(p)); }
  __device__ static __forceinline__ float load_s(const unsigned char* base, int i) {
    return __half2float(reinterpret_cast<const __half*>(base)[i]);
  }
  __device__ static __forceinline__ void mask_neg_inf(uint4& v, uint32_t fl) { mask_neg_inf_u16(v, fl, 0xFC00u); }
};

}  // namespace gr
