// gr_suffix_kv.cu — suffix KV gather of the beam-consecutive attention pass
// for B200 (sm_100a).
//
// The reference copies, for every suffix token of every beam, the token's K
// and V rows (num_heads x head_dim) out of the paged KV cache into contiguous
// buffers with one Triton program per (token, head) and a double indirection
// out -> slot_mapping_out -> slot_mapping -> cache slot
// (vllm_gr/v1/attention/backends/beam_attn.py:62-117).
//
// Here the copy is HBM-bound data movement, laid out for it:
//   * a warp owns 32 output tokens at a time (batches dealt round robin over
//     the grid's warps, CTA-fastest, so the load stays even over the SMs): each
//     lane resolves one token's index chain (two dependent loads), so the 64
//     index loads of the batch are in flight together instead of two round
//     trips per token;
//   * the warp then copies the batch two tokens at a time, K and V rows of both
//     in one unrolled group of 16-byte loads (all issued before the first
//     store), so each lane keeps up to 16 x 16 B in flight;
//   * rows are read through the non-coherent path without L1 allocation and
//     written with plain stores (the attention kernel reads them next, from L2);
//   * a persistent grid of 256-thread CTAs, as many per SM as are resident;
//   * caches whose (head, dim) block is not one contiguous, 16-byte aligned row
//     take an element-wise kernel with the caller's strides.
// Out-of-range sources or slots give zero rows and an error bit (the
// reference reads whatever the address holds).

#include <cstdint>
#include <cuda_runtime.h>
#include <mutex>

#include "../../include/gr_beam.h"
#include "gr_nvtx.h"

namespace grkv {

constexpr int kThreads = 256;
constexpr int kWarps = kThreads / 32;
#ifndef GR_KV_UNROLL
#define GR_KV_UNROLL 4
#endif
constexpr int kUnroll = GR_KV_UNROLL;   // 16-byte vectors per lane per row copy and group

struct Params {
  const unsigned char* k;
  const unsigned char* v;
  const int64_t* slot_mapping;
  const int32_t* slot_mapping_out;
  unsigned char* out_k;
  unsigned char* out_v;
  int32_t* err;
  int64_t num_out, num_src, num_slots;
  int64_t k_tok_bytes, v_tok_bytes;   // token stride in bytes (vector path)
  int nvec;                           // 16-byte vectors per row (vector path)
  int heads, dim, es;
  int64_t ks_tok, ks_head, ks_dim, vs_tok, vs_head, vs_dim;   // element strides (generic path)
};

__device__ __forceinline__ uint4 ld_stream(const uint4* p) {
  uint4 r;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0, %1, %2, %3}, [%4];"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
               : "l"(p));
  return r;
}

// The flat cache slot of output token t, or -1 (and the error bit) when the
// source index or the slot is out of range.
__device__ __forceinline__ int64_t resolve_slot(const Params& P, int64_t t, bool& bad) {
  const int64_t src = static_cast<int64_t>(__ldg(P.slot_mapping_out + t));
  if (src < 0 || src >= P.num_src) {
    bad = true;
    return -1;
  }
  const int64_t slot = __ldg(P.slot_mapping + src);
  if (slot < 0 || slot >= P.num_slots) {
    bad = true;
    return -1;
  }
  return slot;
}

// Output tokens go to warps in batches of 32, round robin over the grid's warps
// numbered CTA-fastest: consecutive batches run on different SMs at once, and a
// grid with more warps than batches leaves its idle warps spread over all SMs.
__device__ __forceinline__ int64_t warp_id_spread() {
  return static_cast<int64_t>(threadIdx.x >> 5) * gridDim.x + blockIdx.x;
}

__global__ void __launch_bounds__(kThreads) gather_rows_kernel(const Params P) {
  const int lane = threadIdx.x & 31;
  const int nvec = P.nvec;
  const uint4 zero = make_uint4(0u, 0u, 0u, 0u);
  const int64_t nwarps = static_cast<int64_t>(gridDim.x) * kWarps;
  for (int64_t t0 = warp_id_spread() * 32; t0 < P.num_out; t0 += nwarps * 32) {
    const int nb = static_cast<int>(min(static_cast<int64_t>(32), P.num_out - t0));
    bool bad = false;
    int64_t slot = -1;
    if (lane < nb) slot = resolve_slot(P, t0 + lane, bad);
    if (__any_sync(0xFFFFFFFFu, bad) && lane == 0 && P.err) atomicOr(P.err, GR_DEVERR_BAD_SLOT);
    for (int i = 0; i < nb; i += 2) {
      const int64_t s0 = __shfl_sync(0xFFFFFFFFu, slot, i);
      const int64_t s1 = __shfl_sync(0xFFFFFFFFu, slot, (i + 1) & 31);
      const bool two = i + 1 < nb;
      const uint4* k0 = reinterpret_cast<const uint4*>(P.k + s0 * P.k_tok_bytes);
      const uint4* v0 = reinterpret_cast<const uint4*>(P.v + s0 * P.v_tok_bytes);
      const uint4* k1 = reinterpret_cast<const uint4*>(P.k + s1 * P.k_tok_bytes);
      const uint4* v1 = reinterpret_cast<const uint4*>(P.v + s1 * P.v_tok_bytes);
      uint4* ok0 = reinterpret_cast<uint4*>(P.out_k) + (t0 + i) * nvec;
      uint4* ov0 = reinterpret_cast<uint4*>(P.out_v) + (t0 + i) * nvec;
      for (int vb = 0; vb < nvec; vb += 32 * kUnroll) {
        uint4 a[kUnroll], b[kUnroll], c[kUnroll], d[kUnroll];
#pragma unroll
        for (int u = 0; u < kUnroll; ++u) {
          const int vi = vb + u * 32 + lane;
          const bool in = vi < nvec;
          a[u] = (in && s0 >= 0) ? ld_stream(k0 + vi) : zero;
          b[u] = (in && s0 >= 0) ? ld_stream(v0 + vi) : zero;
          c[u] = (in && two && s1 >= 0) ? ld_stream(k1 + vi) : zero;
          d[u] = (in && two && s1 >= 0) ? ld_stream(v1 + vi) : zero;
        }
#pragma unroll
        for (int u = 0; u < kUnroll; ++u) {
          const int vi = vb + u * 32 + lane;
          if (vi < nvec) {
            ok0[vi] = a[u];
            ov0[vi] = b[u];
            if (two) {
              ok0[nvec + vi] = c[u];
              ov0[nvec + vi] = d[u];
            }
          }
        }
      }
    }
  }
}

// Element-wise copy with the caller's strides (any (head, dim) layout).
template <typename E>
__global__ void __launch_bounds__(kThreads) gather_elems_kernel(const Params P) {
  const int lane = threadIdx.x & 31;
  const int row = P.heads * P.dim;
  const E* K = reinterpret_cast<const E*>(P.k);
  const E* V = reinterpret_cast<const E*>(P.v);
  E* OK = reinterpret_cast<E*>(P.out_k);
  E* OV = reinterpret_cast<E*>(P.out_v);
  const int64_t nwarps = static_cast<int64_t>(gridDim.x) * kWarps;
  for (int64_t t0 = warp_id_spread() * 32; t0 < P.num_out; t0 += nwarps * 32) {
    const int nb = static_cast<int>(min(static_cast<int64_t>(32), P.num_out - t0));
    bool bad = false;
    int64_t slot = -1;
    if (lane < nb) slot = resolve_slot(P, t0 + lane, bad);
    if (__any_sync(0xFFFFFFFFu, bad) && lane == 0 && P.err) atomicOr(P.err, GR_DEVERR_BAD_SLOT);
    for (int i = 0; i < nb; ++i) {
      const int64_t s = __shfl_sync(0xFFFFFFFFu, slot, i);
      for (int e = lane; e < row; e += 32) {
        const int h = e / P.dim, dd = e - h * P.dim;
        E kx{}, vx{};
        if (s >= 0) {
          kx = K[s * P.ks_tok + h * P.ks_head + dd * P.ks_dim];
          vx = V[s * P.vs_tok + h * P.vs_head + dd * P.vs_dim];
        }
        OK[(t0 + i) * row + e] = kx;
        OV[(t0 + i) * row + e] = vx;
      }
    }
  }
}

// ---- suffix-pass metadata -------------------------------------------------
// One warp per beam of the pass: the beam's request by binary search over the
// records' beam_base, then the beam's stretch of each output array from the
// closed forms of the reference builder's loop (beam_attn.py:319-413): beam 0
// takes min(q_len, remaining + steps) query tokens, every later beam `steps`
// until the request's query budget runs out.
struct MetaParams {
  const gr_suffix_req* reqs;
  int num_reqs;
  int64_t total_beams, total_prefix, total_suffix;
  int64_t* prefix_indices;
  int32_t* smo;
  int32_t* cu_q;
  int32_t* cu_k;
  int32_t* err;
};

__global__ void __launch_bounds__(kThreads) suffix_metadata_kernel(const MetaParams M) {
  const int lane = threadIdx.x & 31;
  const int64_t nwarps = static_cast<int64_t>(gridDim.x) * kWarps;
  if (blockIdx.x == 0 && threadIdx.x == 0) {
    M.cu_q[0] = 0;
    M.cu_k[0] = 0;
  }
  for (int64_t gb = warp_id_spread(); gb < M.total_beams; gb += nwarps) {
    int lo = 0, hi = M.num_reqs - 1;   // last record with beam_base <= gb
    while (lo < hi) {
      const int mid = (lo + hi + 1) >> 1;
      if (static_cast<int64_t>(M.reqs[mid].beam_base) <= gb) lo = mid; else hi = mid - 1;
    }
    const gr_suffix_req R = M.reqs[lo];
    const int64_t b = gb - R.beam_base;
    bool bad = b < 0 || b >= R.beams || R.out_base < 0 || R.suffix_base < 0 || R.remaining < 0 || R.steps < 1 ||
               R.own0 < 1 || R.own_total < R.own0;
    const int64_t extra = static_cast<int64_t>(R.own_total) - R.own0;   // query tokens of beams 1..
    const int64_t before = (b == 0) ? 0 : min((b - 1) * R.steps, extra);
    const int64_t own = (b == 0) ? R.own0 : min(static_cast<int64_t>(R.steps), extra - (b - 1) * R.steps);
    const int64_t q_off = (b == 0) ? 0 : R.own0 + before;
    const int64_t k_off = (b == 0) ? 0 : R.own0 + (b - 1) * R.remaining + before;
    const int64_t seq = (b == 0) ? R.own0 : R.remaining + own;
    bad = bad || own <= 0 || R.out_base + q_off + own > M.total_prefix ||
          R.suffix_base + k_off + seq > M.total_suffix || R.beam_base + b + 1 > M.total_beams;
    if (bad) {
      if (lane == 0 && M.err) atomicOr(M.err, GR_DEVERR_BAD_RECORD);
      continue;
    }
    const int64_t own_start = R.out_base + R.own0 + (b - 1) * R.steps;   // beam b >= 1: its own tokens
    for (int64_t j = lane; j < seq; j += 32) {
      const int64_t val = (b == 0 || j < R.remaining) ? R.out_base + j : own_start + (j - R.remaining);
      M.smo[R.suffix_base + k_off + j] = static_cast<int32_t>(val);
    }
    for (int64_t i = lane; i < own; i += 32) M.prefix_indices[R.out_base + q_off + i] = R.q_start + q_off + i;
    if (lane == 0) {
      M.cu_q[R.beam_base + b + 1] = static_cast<int32_t>(R.out_base + q_off + own);
      M.cu_k[R.beam_base + b + 1] = static_cast<int32_t>(R.suffix_base + k_off + seq);
    }
  }
}

struct Dev {
  int sms = 0;
  int occ_rows = 0;    // resident CTAs per SM of gather_rows_kernel
  int occ_elems = 0;   // of gather_elems_kernel (the 4-byte instance)
};
static Dev g_dev[64];
static std::mutex g_dev_mu;

// The current device's SM count and the kernels' resident CTAs per SM, looked
// up once per device (every entry point of this file uses the same record).
static int device_info(Dev& out) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return GR_ERR_NO_DEVICE;
  std::lock_guard<std::mutex> lock(g_dev_mu);
  if (g_dev[dev].sms == 0) {
    int sms = 0, a = 0, b = 0;
    if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) return GR_ERR_CUDA;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&a, gather_rows_kernel, kThreads, 0) != cudaSuccess ||
        cudaOccupancyMaxActiveBlocksPerMultiprocessor(&b, gather_elems_kernel<uint32_t>, kThreads, 0) != cudaSuccess)
      return GR_ERR_CUDA;
    g_dev[dev].occ_rows = a > 0 ? a : 1;
    g_dev[dev].occ_elems = b > 0 ? b : 1;
    g_dev[dev].sms = sms;
  }
  out = g_dev[dev];
  return GR_OK;
}

}  // namespace grkv

extern "C" int32_t gr_suffix_kv_gather(const gr_kv_gather_desc* d, const void* k_cache, const void* v_cache,
                                       const int64_t* slot_mapping, const int32_t* slot_mapping_out, void* out_k,
                                       void* out_v, int32_t* err, void* stream) {
  gr::NvtxRange nvtx_range("gr_suffix_kv_gather");
  using namespace grkv;
  if (!d) return GR_ERR_NULL;
  if (d->num_out < 0 || d->num_src < 0 || d->num_slots < 0 || d->num_heads <= 0 || d->head_dim <= 0)
    return GR_ERR_BAD_DESC;
  if (d->elem_bytes != 1 && d->elem_bytes != 2 && d->elem_bytes != 4) return GR_ERR_DTYPE;
  if (d->num_out == 0) return GR_OK;
  if (!k_cache || !v_cache || !slot_mapping || !slot_mapping_out || !out_k || !out_v) return GR_ERR_NULL;
  Dev info;
  const int rc = device_info(info);
  if (rc != GR_OK) return rc;
  Params P;
  P.k = static_cast<const unsigned char*>(k_cache);
  P.v = static_cast<const unsigned char*>(v_cache);
  P.slot_mapping = slot_mapping;
  P.slot_mapping_out = slot_mapping_out;
  P.out_k = static_cast<unsigned char*>(out_k);
  P.out_v = static_cast<unsigned char*>(out_v);
  P.err = err;
  P.num_out = d->num_out;
  P.num_src = d->num_src;
  P.num_slots = d->num_slots;
  P.heads = d->num_heads;
  P.dim = d->head_dim;
  P.es = d->elem_bytes;
  P.ks_tok = d->k_stride_tok;
  P.ks_head = d->k_stride_head;
  P.ks_dim = d->k_stride_dim;
  P.vs_tok = d->v_stride_tok;
  P.vs_head = d->v_stride_head;
  P.vs_dim = d->v_stride_dim;
  const int64_t row_bytes = static_cast<int64_t>(d->num_heads) * d->head_dim * d->elem_bytes;
  P.k_tok_bytes = d->k_stride_tok * d->elem_bytes;
  P.v_tok_bytes = d->v_stride_tok * d->elem_bytes;
  P.nvec = static_cast<int>(row_bytes / 16);
  const auto aligned = [](const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; };
  const bool vec = d->k_stride_dim == 1 && d->v_stride_dim == 1 && d->k_stride_head == d->head_dim &&
                   d->v_stride_head == d->head_dim && row_bytes % 16 == 0 && row_bytes / 16 < (1ll << 30) &&
                   P.k_tok_bytes % 16 == 0 && P.v_tok_bytes % 16 == 0 && aligned(k_cache) && aligned(v_cache) &&
                   aligned(out_k) && aligned(out_v);
  // at least ~8 tokens per warp, then every resident CTA
  const int64_t want = (d->num_out + 8 * kWarps - 1) / (8 * kWarps);
  // a persistent grid: every CTA resident at once
  const int64_t cap = static_cast<int64_t>(info.sms) * (vec ? info.occ_rows : info.occ_elems);
  const int grid = static_cast<int>(want < cap ? want : cap);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (vec) {
    gather_rows_kernel<<<grid, kThreads, 0, s>>>(P);
  } else if (d->elem_bytes == 4) {
    gather_elems_kernel<uint32_t><<<grid, kThreads, 0, s>>>(P);
  } else if (d->elem_bytes == 2) {
    gather_elems_kernel<uint16_t><<<grid, kThreads, 0, s>>>(P);
  } else {
    gather_elems_kernel<uint8_t><<<grid, kThreads, 0, s>>>(P);
  }
  return cudaGetLastError() == cudaSuccess ? GR_OK : GR_ERR_CUDA;
}

extern "C" int32_t gr_suffix_metadata(const gr_suffix_req* reqs, int32_t num_reqs, int64_t total_beams,
                                      int64_t total_prefix, int64_t total_suffix, int64_t* prefix_indices,
                                      int32_t* slot_mapping_out, int32_t* cu_seqlens_q, int32_t* cu_seqlens_k,
                                      int32_t* err, void* stream) {
  gr::NvtxRange nvtx_range("gr_suffix_metadata");
  using namespace grkv;
  if (num_reqs < 0 || total_beams < 0 || total_prefix < 0 || total_suffix < 0) return GR_ERR_BAD_DESC;
  if (!cu_seqlens_q || !cu_seqlens_k) return GR_ERR_NULL;
  if ((num_reqs == 0) != (total_beams == 0)) return GR_ERR_BAD_DESC;
  if (total_beams > 0 && (!reqs || !prefix_indices || !slot_mapping_out)) return GR_ERR_NULL;
  Dev info;
  const int rc = device_info(info);
  if (rc != GR_OK) return rc;
  MetaParams M;
  M.reqs = reqs;
  M.num_reqs = num_reqs;
  M.total_beams = total_beams;
  M.total_prefix = total_prefix;
  M.total_suffix = total_suffix;
  M.prefix_indices = prefix_indices;
  M.smo = slot_mapping_out;
  M.cu_q = cu_seqlens_q;
  M.cu_k = cu_seqlens_k;
  M.err = err;
  const int64_t want = (total_beams + kWarps - 1) / kWarps;
  const int64_t cap = static_cast<int64_t>(info.sms) * 4;
  const int grid = static_cast<int>(want < 1 ? 1 : (want < cap ? want : cap));
  suffix_metadata_kernel<<<grid, kThreads, 0, static_cast<cudaStream_t>(stream)>>>(M);
  return cudaGetLastError() == cudaSuccess ? GR_OK : GR_ERR_CUDA;
}

extern "C" int32_t gr_suffix_records(int32_t num_reqs, const int64_t* q_starts, const uint8_t* mega,
                                     const int32_t* prefix_len, const int32_t* cache_len,
                                     const int32_t* beam_width, const int32_t* steps, int32_t block_size,
                                     gr_suffix_req* recs, int64_t* totals) {
  if (num_reqs < 0 || block_size <= 0) return GR_ERR_BAD_DESC;
  if (!totals) return GR_ERR_NULL;
  if (num_reqs > 0 && (!q_starts || !mega || !prefix_len || !cache_len || !beam_width || !steps || !recs))
    return GR_ERR_NULL;
  int64_t n = 0, out_base = 0, suffix_base = 0, beam_base = 0, max_q = 0, max_k = 0;
  for (int32_t i = 0; i < num_reqs; ++i) {
    if (!mega[i]) continue;
    const int64_t plen = prefix_len[i], w = beam_width[i], st = steps[i];
    int64_t clen = cache_len[i], q_offset = 0;
    const int64_t delta = plen - clen;
    if (delta > 0 && delta >= 2 * static_cast<int64_t>(block_size)) {
      // a long uncached prefix runs through standard attention first
      const int64_t std_q = delta < q_starts[i + 1] - q_starts[i] ? delta : q_starts[i + 1] - q_starts[i];
      clen += std_q;
      q_offset = std_q;
    }
    const int64_t q_start = q_starts[i] + q_offset;
    const int64_t q_len = q_starts[i + 1] - q_start;
    if (w == 0 || st == 0 || q_len <= 0) continue;
    const int64_t remaining = plen - clen;
    if (remaining < 0 || w < 0 || st < 0) return GR_ERR_BAD_DESC;
    const int64_t own0 = q_len < remaining + st ? q_len : remaining + st;
    const int64_t room = q_len - own0, full = (w - 1) * st;
    const int64_t extra = room < full ? room : full;
    const int64_t beams = 1 + (extra + st - 1) / st;
    // the records' 32-bit fields must hold these (no silent wrap for large inputs)
    constexpr int64_t kI32Max = 0x7FFFFFFF;
    if (remaining > kI32Max || own0 + extra > kI32Max || beams > kI32Max || beam_base + beams > kI32Max)
      return GR_ERR_BAD_DESC;
    gr_suffix_req& r = recs[n++];
    r.q_start = q_start;
    r.out_base = out_base;
    r.suffix_base = suffix_base;
    r.beam_base = static_cast<int32_t>(beam_base);
    r.beams = static_cast<int32_t>(beams);
    r.remaining = static_cast<int32_t>(remaining);
    r.steps = static_cast<int32_t>(st);
    r.own0 = static_cast<int32_t>(own0);
    r.own_total = static_cast<int32_t>(own0 + extra);
    const int64_t q1 = extra < st ? extra : st;
    if (own0 > max_q) max_q = own0;
    if (q1 > max_q) max_q = q1;
    if (own0 > max_k) max_k = own0;
    if (extra > 0 && remaining + q1 > max_k) max_k = remaining + q1;
    out_base += own0 + extra;
    suffix_base += own0 + (beams - 1) * remaining + extra;
    beam_base += beams;
  }
  totals[0] = n;
  totals[1] = beam_base;
  totals[2] = out_base;
  totals[3] = suffix_base;
  totals[4] = max_q;
  totals[5] = max_k;
  return GR_OK;
}
