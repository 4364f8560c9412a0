// gr_remux.cu — per-request remux of the sampler's logprob rows (sm_100a).
//
// The reference concatenates, in a Python loop over requests, slices of the
// sampler's [rows, K] logprobs / token ids and [rows] ranks into one padded
// row per mega request (vllm_gr/v1/engine/engine_core_patch.py:383-445):
// one slice, reshape, pad and copy per request and tensor, then a cat.  Here
// one launch writes every output row: CTA c owns request c and its threads
// stride over the row's columns, reading the request's sampler rows in order
// (coalesced runs of K) and writing the padding in the same pass.

#include <cstdint>
#include <cuda_runtime.h>

#include "../../include/gr_beam.h"
#include "gr_nvtx.h"

namespace grrx {

constexpr int kThreads = 256;

struct Params {
  const int32_t* row_w;
  const int64_t* row_start;
  const float* lps;
  const unsigned char* ids;
  const unsigned char* ranks;
  const unsigned char* st;
  float* out_lps;
  unsigned char* out_ids;
  unsigned char* out_ranks;
  unsigned char* out_st;
  int64_t max_dim, num_rows, lps_stride, ids_stride, st_stride;
  int K, ids_bytes, ranks_bytes, st_bytes;
};

__device__ __forceinline__ int64_t load_int(const unsigned char* base, int64_t i, int bytes) {
  return bytes == 8 ? reinterpret_cast<const int64_t*>(base)[i]
                    : static_cast<int64_t>(reinterpret_cast<const int32_t*>(base)[i]);
}

__device__ __forceinline__ void store_int(unsigned char* base, int64_t i, int bytes, int64_t v) {
  if (bytes == 8) reinterpret_cast<int64_t*>(base)[i] = v;
  else reinterpret_cast<int32_t*>(base)[i] = static_cast<int32_t>(v);
}

__global__ void __launch_bounds__(kThreads) remux_kernel(const Params P) {
  const int64_t c = blockIdx.x;
  int64_t w = P.row_w[c];
  const int64_t s = P.row_start[c];
  // a request whose rows fall outside the sampler's (inconsistent input) gets a padding row
  if (w < 0 || s < 0 || s + w > P.num_rows || w * P.K > P.max_dim) w = 0;
  const int64_t used = w * P.K;
  const int64_t o = c * P.max_dim;
  for (int64_t j = threadIdx.x; j < P.max_dim; j += kThreads) {
    float lp = -__int_as_float(0x7f800000);
    int64_t id = 0, rk = 0;
    if (j < used) {
      const int64_t r = s + j / P.K, k = j - (j / P.K) * P.K;
      lp = P.lps[r * P.lps_stride + k];
      if (P.ids_bytes) id = load_int(P.ids, r * P.ids_stride + k, P.ids_bytes);
    }
    if (P.ranks_bytes && j < w) rk = load_int(P.ranks, s + j, P.ranks_bytes);
    P.out_lps[o + j] = lp;
    if (P.ids_bytes) store_int(P.out_ids, o + j, P.ids_bytes, id);
    if (P.ranks_bytes) store_int(P.out_ranks, o + j, P.ranks_bytes, rk);
  }
  if (threadIdx.x == 0) store_int(P.out_st, c, P.st_bytes, w > 0 ? load_int(P.st, s * P.st_stride, P.st_bytes) : -1);
}

}  // namespace grrx

extern "C" int32_t gr_remux_logprobs(const gr_remux_desc* d, const int32_t* row_w, const int64_t* row_start,
                                     const float* lps, const void* ids, const void* ranks, const void* st,
                                     float* out_lps, void* out_ids, void* out_ranks, void* out_st, void* stream) {
  gr::NvtxRange nvtx_range("gr_remux_logprobs");
  using namespace grrx;
  if (!d) return GR_ERR_NULL;
  if (d->num_requests < 0 || d->K <= 0 || d->max_dim < 0 || d->num_rows < 0) return GR_ERR_BAD_DESC;
  if ((d->ids_bytes != 0 && d->ids_bytes != 4 && d->ids_bytes != 8) ||
      (d->ranks_bytes != 0 && d->ranks_bytes != 4 && d->ranks_bytes != 8) || (d->st_bytes != 4 && d->st_bytes != 8))
    return GR_ERR_DTYPE;
  if (d->num_requests == 0) return GR_OK;
  if (!row_w || !row_start || !out_lps || !st || !out_st) return GR_ERR_NULL;
  if (d->num_rows > 0 && !lps) return GR_ERR_NULL;
  if ((d->ids_bytes && (!ids || !out_ids)) || (d->ranks_bytes && (!ranks || !out_ranks))) return GR_ERR_NULL;
  Params P;
  P.row_w = row_w;
  P.row_start = row_start;
  P.lps = lps;
  P.ids = static_cast<const unsigned char*>(ids);
  P.ranks = static_cast<const unsigned char*>(ranks);
  P.st = static_cast<const unsigned char*>(st);
  P.out_lps = out_lps;
  P.out_ids = static_cast<unsigned char*>(out_ids);
  P.out_ranks = static_cast<unsigned char*>(out_ranks);
  P.out_st = static_cast<unsigned char*>(out_st);
  P.max_dim = d->max_dim;
  P.num_rows = d->num_rows;
  P.lps_stride = d->lps_stride;
  P.ids_stride = d->ids_stride;
  P.st_stride = d->st_stride;
  P.K = d->K;
  P.ids_bytes = d->ids_bytes;
  P.ranks_bytes = d->ranks_bytes;
  P.st_bytes = d->st_bytes;
  remux_kernel<<<d->num_requests, kThreads, 0, static_cast<cudaStream_t>(stream)>>>(P);
  return cudaGetLastError() == cudaSuccess ? GR_OK : GR_ERR_CUDA;
}
