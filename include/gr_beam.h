/*
 * gr_beam.h — C ABI of the B200-native constrained beam-search step.
 *
 * One call of gr_beam_step() advances R beam-search requests by one decode
 * step.  For every request it
 *   1. takes each beam's next-token logits row (bf16 / f16 / f32),
 *   2. normalises it over the whole vocabulary in vLLM's log-prob domain
 *      (raw: log_softmax(x); processed: log_softmax(penalise(x) / T)),
 *   3. restricts each beam to its candidate tokens: the children of its node
 *      in the item-catalog trie (CSR), or all tokens for an unconstrained beam,
 *      or (reference-literal mode) the beam's own top-K tokens with the
 *      disallowed ones set to -inf,
 *   4. adds the beam's cumulative score, moves EOS candidates out of the pool,
 *   5. selects the top 2*beam_width (token, parent) candidates of the request
 *      in canonical order: score descending, then flat index parent*V+token
 *      ascending,
 *   6. emits the first beam_width of them as the new beams together with the
 *      child trie node and the forked per-beam token table.
 *
 * It replaces, as one device call, the per-step work of the reference
 * (vLLM-GR) that is spread over:
 *   - vLLM Sampler.forward -> compute_logprobs / gather_logprobs
 *     (vllm v1/sample/sampler.py:67-140, 300-352; penalties :366-433),
 *   - vllm_gr/logprobs.py:34-53           extract_and_dedup_flat_logprobs,
 *   - vllm_gr/entrypoints/openai/serving_models.py:42-49  Catalog.valid,
 *   - vllm_gr/entrypoints/openai/serving_engine.py:457-597 (mask, cum add,
 *     EOS -> completed, argpartition top-B, new beams, fork_info),
 *   - vllm_gr/entrypoints/llm.py:201-280   (same selection, offline),
 *   - vllm_gr/csrc/minheap.cpp:75-114      (striped bounded top-N).
 *
 * Conventions
 *   - Every pointer is a device pointer unless stated otherwise.  The caller
 *     owns (allocates and frees) every buffer, including the workspace; the
 *     library allocates no device memory.
 *   - Calls are stream ordered and never synchronise the host.  `stream` is a
 *     cudaStream_t passed as void* (NULL = the legacy default stream).
 *   - Return value 0 = success, negative = gr_status error.  No call aborts,
 *     throws or traps.  Errors found on the device (bad node id, CSR child
 *     token out of range, a bounded wait that ran out) are OR-ed into the
 *     caller's device error word io->err as GR_DEVERR_* bits.
 *   - The workspace must be at least gr_beam_step_workspace_size() bytes and
 *     256-byte aligned.  Its contents need not be initialised.
 *   - Calls that share a workspace must not overlap on the GPU.
 */
#ifndef GR_BEAM_H_
#define GR_BEAM_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define GR_ABI_VERSION 2

typedef enum gr_status {
  GR_OK = 0,
  GR_ERR_NULL = -1,          /* a required pointer is NULL                    */
  GR_ERR_BAD_DESC = -2,      /* sizes / ids out of range or inconsistent      */
  GR_ERR_DTYPE = -3,         /* unsupported logit dtype or logprobs mode      */
  GR_ERR_MISALIGNED = -4,    /* workspace not 256-byte aligned                */
  GR_ERR_WORKSPACE = -5,     /* workspace smaller than required               */
  GR_ERR_UNSUPPORTED = -6,   /* valid request outside this build's limits     */
  GR_ERR_CUDA = -7,          /* a CUDA runtime call or launch failed          */
  GR_ERR_NO_DEVICE = -8      /* no sm_100 device is current                   */
} gr_status;

/* Bits OR-ed into *io->err by the kernels. */
#define GR_DEVERR_BAD_NODE      0x1   /* node id outside [-2, num_nodes)        */
#define GR_DEVERR_BAD_CHILD     0x2   /* CSR child token outside [0, vocab)     */
#define GR_DEVERR_TIMEOUT       0x4   /* a bounded mbarrier wait ran out        */
#define GR_DEVERR_OVERFLOW      0x8   /* per-request candidate buffer overflow  */
#define GR_DEVERR_TIE_BOUNDARY  0x10  /* reserved: no longer raised (a streamed
                                         top-k whose boundary could tie a dropped
                                         column is recomputed exactly)          */

typedef enum gr_dtype {
  GR_DTYPE_F32 = 0,
  GR_DTYPE_BF16 = 1,
  GR_DTYPE_F16 = 2
} gr_dtype;

/* vLLM LogprobsMode (vllm config/model.py): "raw_logprobs" is log_softmax of
 * the raw logits, "processed_logprobs" is log_softmax after penalties and
 * temperature (vllm v1/sample/sampler.py:80-88, 223-233, 262-265). */
typedef enum gr_logprobs_mode {
  GR_LOGPROBS_RAW = 0,
  GR_LOGPROBS_PROCESSED = 1
} gr_logprobs_mode;

/* Node id conventions for io->node / sel_node. */
#define GR_NODE_UNCONSTRAINED (-1)  /* every vocab token is a candidate       */
#define GR_NODE_DEAD (-2)           /* prefix not in the catalog: no children */

typedef struct gr_step_desc {
  int32_t num_requests;   /* R                                                */
  int32_t num_beams;      /* beam rows per request in this step (>= 1)        */
  int32_t beam_width;     /* B: beams kept; 2*B candidates are emitted        */
  int32_t vocab_size;     /* V: full vocabulary (token ids are in [0, V))     */
  int32_t vocab_local;    /* columns present in `logits` (== V unsharded)     */
  int32_t vocab_offset;   /* token id of column 0 (0 unsharded)               */
  int64_t row_stride;     /* elements between consecutive logit rows          */
  int32_t logit_dtype;    /* gr_dtype                                         */
  int32_t logprobs_mode;  /* gr_logprobs_mode                                 */
  int32_t per_beam_k;     /* 0: all allowed children are candidates;
                             K>0: reference-literal, each beam's raw top-K
                             (after the sampled-token dedup) then masked      */
  int32_t eos_token_id;   /* -1: no EOS handling (ignore_eos)                 */
  int32_t hist_len;       /* T: tokens per beam in hist_in (fork table and,
                             in processed mode, the penalty history)          */
  int32_t num_nodes;      /* N: CSR trie nodes (0 if no catalog)              */
  int64_t num_edges;      /* E: CSR trie edges                                */
  int32_t vocab_stride;   /* local column j holds token vocab_offset +
                             j * vocab_stride (0 or 1: a contiguous slice;
                             S with vocab_offset = k: shard k of a strided
                             split over S ranks, tokens k, k + S, ...)      */
  int32_t flags;          /* GR_STEP_* bits (0: none)                         */
} gr_step_desc;

/* gr_step_desc.flags (gr_beam_step / gr_beam_step_noalloc; the vocab-sharded
 * entry points take 0).  GR_STEP_CLEAR_ERR: the step sets *io->err to 0
 * before any of its kernels reports into it, so the caller need not zero the
 * word first (one launch less per step); without it device errors are OR-ed
 * into the word as it stands. */
#define GR_STEP_CLEAR_ERR 0x1

typedef struct gr_step_io {
  /* inputs */
  const void* logits;          /* [R*num_beams rows][row_stride], dtype desc  */
  const float* cum;            /* [R*num_beams] cumulative beam scores        */
  const int32_t* node;         /* [R*num_beams] trie node of each beam        */
  const int64_t* row_ptr;      /* [N+1] CSR offsets (may be NULL if N == 0)   */
  const int32_t* child_tok;    /* [E] child token ids, ascending per node     */
  const int32_t* child_node;   /* [E] child node ids                          */
  const float* temperature;    /* [R] or NULL (= 1); T < 1e-5 means 1         */
  const float* rep_penalty;    /* [R] or NULL (= 1)                           */
  const float* pres_penalty;   /* [R] or NULL (= 0)                           */
  const float* freq_penalty;   /* [R] or NULL (= 0)                           */
  const int32_t* hist_in;      /* [R*num_beams][T] generated tokens, or NULL
                                  when T == 0; entries < 0 are padding        */
  /* outputs (all required unless marked optional) */
  float* cand_score;           /* [R][2B] sorted canonical candidates         */
  int32_t* cand_token;         /* [R][2B]  (-1 padding)                       */
  int32_t* cand_parent;        /* [R][2B]  (-1 padding)                       */
  float* sel_score;            /* [R][B] new cumulative scores                */
  int32_t* sel_token;          /* [R][B]                                      */
  int32_t* sel_parent;         /* [R][B] parent beam index within request     */
  int32_t* sel_node;           /* [R][B] child trie node (-1/-2 as above)     */
  float* eos_score;            /* [R*num_beams] cum+lp of the beam's EOS
                                  candidate, NaN if it had none (optional)    */
  int32_t* hist_out;           /* [R][B][T+1] forked token table (optional)   */
  float* lse;                  /* [R*num_beams] row log-sum-exp (optional)    */
  int32_t* err;                /* device error word, GR_DEVERR_* bits         */
} gr_step_io;

/* Library ABI version (GR_ABI_VERSION). */
int32_t gr_abi_version(void);

/* Human-readable name of a gr_status value (static string). */
const char* gr_status_string(int32_t status);

/* Bytes of workspace gr_beam_step() needs for `desc`.
 * Replaces nothing in the reference (the reference allocates per step in
 * Python lists / NumPy arrays: serving_engine.py:457-535). */
int32_t gr_beam_step_workspace_size(const gr_step_desc* desc, size_t* bytes);

/* One constrained beam-search step for all requests (see top of file).
 * Replaces: vllm v1/sample/sampler.py:67-140 (logprobs) +
 * vllm_gr/logprobs.py:34-53 + serving_engine.py:457-597 / llm.py:201-280. */
int32_t gr_beam_step(const gr_step_desc* desc, const gr_step_io* io,
                     void* workspace, size_t workspace_bytes, void* stream);

/* Size of the device scratch built into the library for gr_beam_step_noalloc. */
#define GR_NOALLOC_SCRATCH_BYTES (16u << 20)

/* The same step as gr_beam_step, for callers that cannot allocate device
 * memory (for example code running where a cudaMalloc would synchronise the
 * device or break a memory pool's accounting, or hosts with no allocator of
 * their own): it takes no workspace and allocates nothing.  It uses a fixed
 * GR_NOALLOC_SCRATCH_BYTES array of device memory that the library holds on
 * every GPU it is loaded on, until the process exits.
 *   - Requests whose gr_beam_step_workspace_size exceeds that size are
 *     rejected with GR_ERR_WORKSPACE (use gr_beam_step with your own
 *     workspace for them).
 *   - The first call on a device looks up the array's device address (with
 *     that device current); make that first call before any stream capture.
 *   - All calls share the one array: calls that may run at the same time on
 *     the GPU (different streams, different host threads) race on it and must
 *     be serialised by the caller.
 *   - The address is kept for the life of the process: the library must not
 *     be used across a reset of the device (cudaDeviceReset) that would move
 *     or free the array.
 * No counterpart in the reference (an addition of this library). */
int32_t gr_beam_step_noalloc(const gr_step_desc* desc, const gr_step_io* io, void* stream);

/* ---- vocab-sharded lm_head (logit columns split over ranks) --------------
 *
 * With the lm_head split by vocabulary columns, shard k holds the columns of
 * tokens vocab_offset + j * vocab_stride, j < vocab_local, of every row (vLLM
 * would all-gather the full logits first: vllm logits_processor.py:75-86):
 * a contiguous slice (vocab_stride 1) or, with the lm_head's weight rows
 * dealt round robin once at load time, a strided split (vocab_offset = k,
 * vocab_stride = number of shards).  The strided split gives every shard
 * about 1/S of each trie node's children, which sit in one contiguous token
 * range (semantic-ID codebooks at the vocabulary's tail), so the candidate
 * work is balanced.  A step becomes three calls with two all-gathers between
 * them, all on the caller's stream; every call takes the gr_beam_step
 * workspace (same size).
 *
 * Phase 1 (every shard): per-row partial (max, sum exp(y - max)) over the
 * local columns, y the log-prob domain value (processed mode: penalties and
 * temperature applied), written to partials[row][2] = {max, sumexp}.
 * Replaces the full-row log_softmax of vllm sampler.py:300-301.
 */
int32_t gr_lse_partials(const gr_step_desc* desc, const gr_step_io* io, float* partials,
                        void* workspace, size_t workspace_bytes, void* stream);

/* Phase 2 (every shard, after the caller all-gathered the partials of all
 * `num_shards` shards into gathered_partials[num_shards][R*num_beams][2]):
 * combines them into the rows' global lse (written to io->lse when it is not
 * NULL), scores this shard's catalog children and writes the shard's
 * top-2B keys per request to shard_keys[R][2B] in canonical order (key
 * descending: score, then lower flat index parent*V+token), zero padded.
 * The keys are the same bytes on every run and for every kernel choice.
 * io->eos_score is valid on the shard whose columns hold eos_token_id.
 * Constrained (per_beam_k == 0) steps only. */
int32_t gr_shard_candidates(const gr_step_desc* desc, const gr_step_io* io,
                            const float* gathered_partials, int32_t num_shards,
                            uint64_t* shard_keys, void* workspace,
                            size_t workspace_bytes, void* stream);

/* Phase 3 (every shard, after the caller all-gathered shard_keys of all
 * shards into gathered_keys[num_shards][R][2B]): merges them into the global
 * top-2B per request and writes cand_* / sel_* / sel_node / hist_out of `io`
 * (the logits field is unused).  Every shard computes the same result. */
int32_t gr_merge_candidates(const gr_step_desc* desc, const gr_step_io* io,
                            const uint64_t* gathered_keys, int32_t num_shards,
                            void* workspace, size_t workspace_bytes, void* stream);

/* ---- suffix KV gather for the beam-consecutive attention pass -------------
 *
 * The beams of a mega-request attend to the shared prefix through the paged
 * KV cache and to their own suffix (the uncached prefix tail plus the tokens
 * decoded since the fork) through a contiguous copy.  This gathers that copy:
 * for every output token t
 *     src  = slot_mapping_out[t]                       (index into slot_mapping)
 *     slot = slot_mapping[src]                         (flat cache slot)
 *     out_k[t, h, d] = k_cache[slot * k_stride_tok + h * k_stride_head + d * k_stride_dim]
 * and the same for V.  Strides are in elements; out_k / out_v are contiguous
 * [num_out][num_heads][head_dim].  A flat slot is block * block_size + offset
 * (vLLM's layout with the blocks contiguous, so the token stride applies).
 * Sources outside [0, num_src) or slots outside [0, num_slots) produce zero
 * rows and set GR_DEVERR_BAD_SLOT in *err (err may be NULL).
 * Replaces vllm_gr/v1/attention/backends/beam_attn.py:62-117
 * (paged_kv_to_contig_suffix_kernel, extract_suffix_kv). */
#define GR_DEVERR_BAD_SLOT      0x20  /* suffix gather: source or slot out of range */

typedef struct gr_kv_gather_desc {
  int64_t num_out;          /* output tokens (slot_mapping_out entries)          */
  int64_t num_src;          /* slot_mapping entries                              */
  int64_t num_slots;        /* cache slots (num_blocks * block_size)             */
  int32_t num_heads;        /* KV heads                                          */
  int32_t head_dim;         /* elements per head                                 */
  int32_t elem_bytes;       /* 1, 2 or 4                                         */
  int32_t reserved;
  int64_t k_stride_tok, k_stride_head, k_stride_dim;
  int64_t v_stride_tok, v_stride_head, v_stride_dim;
} gr_kv_gather_desc;

int32_t gr_suffix_kv_gather(const gr_kv_gather_desc* desc, const void* k_cache, const void* v_cache,
                            const int64_t* slot_mapping, const int32_t* slot_mapping_out,
                            void* out_k, void* out_v, int32_t* err, void* stream);

/* Suffix-pass metadata of mega-decode requests, built on the device.
 *
 * The host keeps the per-request arithmetic of the reference builder (O(1) per
 * request) and passes one record per request that takes part in the pass, in
 * request order (`reqs` is a device array).  The call writes the per-beam and
 * per-token arrays the reference builds in Python loops
 * (beam_attn.py:319-413, 432-476).  With own_b the query tokens of beam b
 * (own_0 = own0; for b >= 1 min(steps, own_total - own0 - (b-1)*steps)) and
 * its suffix length seq_b (own0 for beam 0, remaining + own_b otherwise):
 *   prefix_indices[out_base + i] = q_start + i                 for i < own_total
 *   slot_mapping_out[suffix_base + sum_{c<b} seq_c + j]       for j < seq_b:
 *       beam 0:  out_base + j
 *       beam b:  out_base + j                                    (j < remaining)
 *                out_base + own0 + (b-1)*steps + (j - remaining) (otherwise)
 *   cu_seqlens_q[beam_base + b + 1] = out_base + sum_{c<=b} own_c
 *   cu_seqlens_k[beam_base + b + 1] = suffix_base + sum_{c<=b} seq_c
 *   cu_seqlens_q[0] = cu_seqlens_k[0] = 0
 * out_base / suffix_base / beam_base are the running totals of own_total /
 * sum seq / beams over the earlier records.  Replaces, for the suffix pass,
 * BeamAttentionMetadataBuilder._build_mega_mappings and the tensors made from
 * its lists in _create_mega_tensors. */
typedef struct gr_suffix_req {
  int64_t q_start;       /* first query token of the request's mega part         */
  int64_t out_base;      /* its first position in the mega token order             */
  int64_t suffix_base;   /* its first entry in slot_mapping_out                    */
  int32_t beam_base;     /* its first beam in the cu_seqlens arrays                */
  int32_t beams;         /* active beams (beam 0 included), >= 1                   */
  int32_t remaining;     /* uncached prefix tokens (beam 0's first ones)           */
  int32_t steps;         /* decode steps per beam, >= 1                            */
  int32_t own0;          /* beam 0's query tokens, >= 1                            */
  int32_t own_total;     /* all query tokens of the request's mega part            */
} gr_suffix_req;

/* Host helper (no device, no allocation): the records of gr_suffix_metadata
 * from the reference builder's per-request inputs, all host arrays of length
 * num_reqs (mega[i] = 0 marks a standard request; q_starts has num_reqs + 1
 * entries).  Writes at most num_reqs records to `recs` and the totals
 * (records, beams, prefix tokens, suffix tokens, max query / suffix length of
 * a beam) to totals[6].  Follows beam_attn.py:255-292 (a long uncached prefix
 * first goes through standard attention) and 319-413 (beam 0's share, then
 * `steps` per beam until the query budget runs out).  GR_ERR_BAD_DESC when a
 * request's cache_len exceeds its prefix_len after that split, or when a
 * record's field (uncached tokens, query tokens, beams, the running beam
 * count) would not fit in 32 bits. */
int32_t gr_suffix_records(int32_t num_reqs, const int64_t* q_starts, const uint8_t* mega,
                          const int32_t* prefix_len, const int32_t* cache_len, const int32_t* beam_width,
                          const int32_t* steps, int32_t block_size, gr_suffix_req* recs, int64_t* totals);

#define GR_DEVERR_BAD_RECORD    0x40  /* suffix metadata: a record points outside the outputs */

/* prefix_indices has total_prefix entries, slot_mapping_out total_suffix, the
 * cu_seqlens arrays total_beams + 1.  Writes a record would place outside them
 * are dropped and set GR_DEVERR_BAD_RECORD in *err (err may be NULL). */
int32_t gr_suffix_metadata(const gr_suffix_req* reqs, int32_t num_reqs, int64_t total_beams,
                           int64_t total_prefix, int64_t total_suffix, int64_t* prefix_indices,
                           int32_t* slot_mapping_out, int32_t* cu_seqlens_q, int32_t* cu_seqlens_k,
                           int32_t* err, void* stream);

/* ---- logprobs remux of mega requests (worker side) -----------------------
 *
 * vLLM's sampler returns K logprobs (and token ids) per logit row and one
 * rank per row; a mega request owns `row_w[c]` consecutive rows (0 for a
 * chunked prefill that produced none).  Per request c this writes one row:
 *   out_lps[c][j]   = lps[(row_start[c] + j / K) * lps_stride + j % K]   j < row_w*K, else -inf
 *   out_ids[c][j]   = ids[... same ...]                                   else 0
 *   out_ranks[c][j] = ranks[row_start[c] + j]                              j < row_w, else 0
 *   out_st[c]       = st[row_start[c] * st_stride]                         row_w > 0, else -1
 * for j < max_dim.  Integer arrays are 4- or 8-byte (ids_bytes / ranks_bytes
 * 0 = the array is absent).  row_w and row_start are device arrays.
 * Replaces vllm_gr/v1/engine/engine_core_patch.py:383-445
 * (_remux_logprobs_tensors: a Python loop of slices, pads and one cat). */
typedef struct gr_remux_desc {
  int32_t num_requests;
  int32_t K;                 /* logprob columns taken per row (<= the rows' width) */
  int64_t max_dim;           /* output row width (>= max row_w * K)                 */
  int64_t num_rows;          /* sampler rows                                        */
  int64_t lps_stride;        /* elements between sampler rows of lps / ids          */
  int64_t ids_stride;
  int64_t st_stride;         /* elements between rows of st                         */
  int32_t ids_bytes;         /* 0, 4 or 8                                           */
  int32_t ranks_bytes;       /* 0, 4 or 8                                           */
  int32_t st_bytes;          /* 4 or 8                                              */
  int32_t reserved;
} gr_remux_desc;

int32_t gr_remux_logprobs(const gr_remux_desc* desc, const int32_t* row_w, const int64_t* row_start,
                          const float* lps, const void* ids, const void* ranks, const void* st,
                          float* out_lps, void* out_ids, void* out_ranks, void* out_st, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* GR_BEAM_H_ */
