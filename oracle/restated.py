"""CPU oracle: a NumPy restatement of the reference's constrained beam step.

TEST INFRASTRUCTURE ONLY.  Nothing in the product path imports this module;
only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline / reference
legs use it, and only as the checker or as the timed CPU baseline.

What it restates (reference = vLLM-GR, sampler = the vLLM version it runs on):
  * log-prob domain, vLLM v1 Sampler:
      raw:        lp = log_softmax(float32(x))            (sampler.py:300-301)
      processed:  lp = log_softmax(penalise(x) / T)       (sampler.py:223-233,
                  262-265; model_executor/layers/utils.py:51-89)
    penalise():   repetition  x>0 ? x/rep : x*rep on tokens seen
                  frequency   x -= freq * count
                  presence    x -= pres * (count > 0)
    temperature:  T < 1e-5 is treated as 1 (sampler.py apply_temperature)
  * per-beam candidate list:
      constrained (per_beam_k == 0): the children of the beam's trie node —
        the set Catalog.valid(prefix) returns (serving_models.py:42-49);
      unconstrained (node == -1): every token;
      reference-literal (per_beam_k = K): vLLM's flat logprobs
        [sampled, top1..topK] (sampler.py:304-352) de-duplicated by
        extract_and_dedup_flat_logprobs (vllm_gr/logprobs.py:34-53), then
        tokens outside the catalog set to -inf (serving_engine.py:504-506,
        526-528).  `sampled` is the greedy token: argmax of the penalised
        logits, lowest index on ties.
  * score = cum + lp (serving_engine.py:511, 533; llm.py:218-220)
  * EOS candidates are recorded as completions and set to -inf in the pool
    (serving_engine.py:541-562; llm.py:233-254)
  * selection: the reference takes argpartition(-score, B)[:B] in an
    unspecified order (serving_engine.py:566-569; llm.py:256-262).  This
    oracle returns the top 2*B in the canonical order (score descending, then
    flat index parent*V + token ascending); its first B entries are the
    reference's top-B up to ties.
  * new beams: parent index, token, child trie node, and the forked token
    table hist_out[i] = hist_in[parent_i] + [token_i]
    (serving_engine.py:571-590 fork_info; llm.py:263-276).

Two arithmetic modes:
  'reference'  lp32 = float32(y - lse) with lse in float64, and the score
               summed in float64 as the reference does with Python floats.
  'device'     lse32 given (or float32(lse64)); lp32 = f32(y32 - lse32);
               score32 = f32(cum32 + lp32) — the rounding the CUDA step uses,
               so that selection can be checked bit for bit given its lse.
"""
from __future__ import annotations

import numpy as np

RAW = 0
PROCESSED = 1
NODE_UNCONSTRAINED = -1
NODE_DEAD = -2
_SAMPLING_EPS = 1e-5


# --------------------------------------------------------------------------
# dtype helpers
# --------------------------------------------------------------------------
def bf16_bits_to_f32(bits: np.ndarray) -> np.ndarray:
    """uint16 bfloat16 bit patterns -> float32 (exact)."""
    return (bits.astype(np.uint32) << 16).view(np.float32)


def f32_to_bf16_bits(x: np.ndarray) -> np.ndarray:
    """float32 -> bfloat16 bits, round to nearest even (what torch .to(bf16) does)."""
    u = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32).astype(np.uint64)
    rounding = ((u >> 16) & 1) + 0x7FFF
    out = ((u + rounding) >> 16).astype(np.uint16)
    nan = np.isnan(x)
    if nan.any():
        out[nan] = 0x7FC0
    return out


# --------------------------------------------------------------------------
# log-prob domain
# --------------------------------------------------------------------------
def effective_temperature(t: float) -> np.float32:
    t = np.float32(t)
    return np.float32(1.0) if t < _SAMPLING_EPS else t


def penalise_row(x32: np.ndarray, hist_row, vocab_offset: int,
                 rep: float, pres: float, freq: float) -> np.ndarray:
    """vLLM apply_penalties restricted to one row (float32, IEEE order).

    Follows model_executor/layers/utils.py:51-89 and the repetition op
    (_custom_ops.py:360-373): repetition first, then frequency, then presence,
    each rounded to float32.  Only tokens in the history change."""
    out = np.array(x32, dtype=np.float32, copy=True)
    if hist_row is None or len(hist_row) == 0:
        return out
    h = np.asarray(hist_row, dtype=np.int64)
    h = h[h >= 0] - vocab_offset
    h = h[(h >= 0) & (h < out.shape[0])]
    if h.size == 0:
        return out
    uniq, counts = np.unique(h, return_counts=True)
    xv = out[uniq]
    rep32 = np.float32(rep)
    xv = np.where(xv > 0, xv / rep32, xv * rep32).astype(np.float32)
    xv = (xv - (np.float32(freq) * counts.astype(np.float32)).astype(np.float32)).astype(np.float32)
    xv = (xv - np.float32(pres)).astype(np.float32)
    out[uniq] = xv
    return out


def has_penalties(rep, pres, freq) -> bool:
    return not (np.float32(rep) == 1 and np.float32(pres) == 0 and np.float32(freq) == 0)


def processed_row(x32, hist_row, vocab_offset, temp, rep, pres, freq):
    """penalise(x) / T in float32 (sampler.py:223-233 then apply_temperature)."""
    y = penalise_row(x32, hist_row, vocab_offset, rep, pres, freq) if has_penalties(rep, pres, freq) \
        else np.array(x32, dtype=np.float32, copy=True)
    t = effective_temperature(temp)
    if t != np.float32(1.0):
        y = (y / t).astype(np.float32)
    return y


def lse64(y32: np.ndarray) -> float:
    y = y32.astype(np.float64)
    m = np.max(y)
    if not np.isfinite(m):
        return float(m)
    return float(m + np.log(np.sum(np.exp(y - m))))


# --------------------------------------------------------------------------
# canonical top-k helpers
# --------------------------------------------------------------------------
def canonical_order(scores: np.ndarray, flat: np.ndarray) -> np.ndarray:
    """Indices sorting by score descending, then flat index ascending."""
    return np.lexsort((flat, -scores.astype(np.float64)))


def topk_canonical(scores: np.ndarray, flat: np.ndarray, k: int) -> np.ndarray:
    """Indices of the canonical top-k (score desc, flat asc), sorted."""
    n = scores.shape[0]
    if n <= k:
        return canonical_order(scores, flat)
    s64 = scores.astype(np.float64)
    kth = np.partition(-s64, k - 1)[k - 1]          # -(k-th largest score)
    keep = np.nonzero(-s64 <= kth)[0]               # every score >= k-th, ties included
    order = canonical_order(s64[keep], flat[keep])
    return keep[order[:k]]


# --------------------------------------------------------------------------
# CSR trie helpers
# --------------------------------------------------------------------------
class CSR:
    def __init__(self, row_ptr, child_tok, child_node):
        self.row_ptr = np.asarray(row_ptr, dtype=np.int64)
        self.child_tok = np.asarray(child_tok, dtype=np.int32)
        self.child_node = np.asarray(child_node, dtype=np.int32)

    @property
    def num_nodes(self):
        return int(self.row_ptr.shape[0] - 1)

    def children(self, n: int):
        a, b = self.row_ptr[n], self.row_ptr[n + 1]
        return self.child_tok[a:b], self.child_node[a:b]

    def child_of(self, n: int, tok: int) -> int:
        """Trie step: node reached from n by tok (-1 stays -1, dead = -2)."""
        if n == NODE_UNCONSTRAINED:
            return NODE_UNCONSTRAINED
        if n < 0:
            return NODE_DEAD
        toks, nodes = self.children(n)
        i = np.searchsorted(toks, tok)
        if i < toks.shape[0] and toks[i] == tok:
            return int(nodes[i])
        return NODE_DEAD


# --------------------------------------------------------------------------
# the step
# --------------------------------------------------------------------------
def beam_step(logits32: np.ndarray, cum: np.ndarray, node: np.ndarray, csr: CSR | None,
              *, beam_width: int, vocab_size: int | None = None, vocab_offset: int = 0,
              logprobs_mode: int = RAW, per_beam_k: int = 0, eos_token_id: int = -1,
              hist_in: np.ndarray | None = None, temperature=None, rep_penalty=None,
              pres_penalty=None, freq_penalty=None, arith: str = "reference",
              lse_override: np.ndarray | None = None) -> dict:
    """One step for R requests.

    logits32: float32 [R, NB, V_l] (bf16 inputs converted exactly first)
    cum: float32 [R, NB]; node: int32 [R, NB]; hist_in: int32 [R, NB, T] or None
    temperature / penalties: per-request sequences of length R or None.
    Returns the same outputs as the CUDA step (see include/gr_beam.h)."""
    logits32 = np.asarray(logits32, dtype=np.float32)
    R, NB, VL = logits32.shape
    V = int(vocab_size if vocab_size is not None else VL)
    B = int(beam_width)
    K2 = 2 * B
    cum = np.asarray(cum, dtype=np.float32).reshape(R, NB)
    node = np.asarray(node, dtype=np.int32).reshape(R, NB)
    T = 0 if hist_in is None else int(hist_in.shape[-1])
    if hist_in is not None:
        hist_in = np.asarray(hist_in, dtype=np.int32).reshape(R, NB, T)

    def per_req(a, default):
        return [default] * R if a is None else [float(v) for v in np.asarray(a).reshape(R)]

    temps = per_req(temperature, 1.0)
    reps = per_req(rep_penalty, 1.0)
    press = per_req(pres_penalty, 0.0)
    freqs = per_req(freq_penalty, 0.0)

    out = {
        "cand_score": np.full((R, K2), -np.inf, np.float32),
        "cand_token": np.full((R, K2), -1, np.int32),
        "cand_parent": np.full((R, K2), -1, np.int32),
        "sel_score": np.full((R, B), -np.inf, np.float32),
        "sel_token": np.full((R, B), -1, np.int32),
        "sel_parent": np.full((R, B), -1, np.int32),
        "sel_node": np.full((R, B), NODE_DEAD, np.int32),
        "eos_score": np.full((R, NB), np.nan, np.float32),
        "hist_out": np.full((R, B, T + 1), -1, np.int32),
        "lse": np.zeros((R, NB), np.float32),
        "cand_score64": np.full((R, K2), -np.inf, np.float64),
    }

    for r in range(R):
        pool_s, pool_f = [], []
        for b in range(NB):
            x = logits32[r, b]
            hrow = None if hist_in is None else hist_in[r, b]
            pen = has_penalties(reps[r], press[r], freqs[r])
            if logprobs_mode == PROCESSED:
                y = processed_row(x, hrow, vocab_offset, temps[r], reps[r], press[r], freqs[r])
            else:
                y = np.array(x, dtype=np.float32, copy=True)
            l64 = lse64(y)
            if lse_override is not None:
                l32 = np.float32(np.asarray(lse_override).reshape(R, NB)[r, b])
            else:
                l32 = np.float32(l64)
            out["lse"][r, b] = l32

            def lp_of(idx):
                """float32 log-probs of local columns idx."""
                if arith == "device":
                    return (y[idx] - l32).astype(np.float32)
                return (y[idx].astype(np.float64) - l64).astype(np.float32)

            def score_of(lp32):
                if arith == "device":
                    return (np.float32(cum[r, b]) + lp32).astype(np.float32).astype(np.float64)
                return np.float64(cum[r, b]) + lp32.astype(np.float64)

            n = int(node[r, b])
            if n < NODE_DEAD or (csr is not None and n >= csr.num_nodes) or (csr is None and n >= 0):
                raise ValueError(f"bad node id {n}")

            if per_beam_k > 0:
                # reference-literal: vLLM top-K over the whole (local) vocab
                K = per_beam_k
                if K > VL:
                    raise ValueError("per_beam_k larger than the vocabulary")
                lp_all = lp_of(np.arange(VL))
                toks = np.arange(VL, dtype=np.int64) + vocab_offset
                top = topk_canonical(lp_all.astype(np.float64), toks, K)
                top_tok = toks[top]
                # sampled token: greedy argmax of the penalised logits
                xs = penalise_row(x, hrow, vocab_offset, reps[r], press[r], freqs[r]) if pen else x
                sampled = int(np.argmax(xs)) + vocab_offset
                if sampled in set(top_tok.tolist()):
                    cand_tok = top_tok
                else:
                    cand_tok = np.concatenate([[sampled], top_tok[:K - 1]])
                lp = lp_of(cand_tok - vocab_offset)
                if n >= 0:
                    allowed = set(csr.children(n)[0].tolist())
                    ok = np.array([t in allowed for t in cand_tok.tolist()], dtype=bool)
                elif n == NODE_DEAD:
                    ok = np.zeros(cand_tok.shape[0], dtype=bool)
                else:
                    ok = np.ones(cand_tok.shape[0], dtype=bool)
                sc = np.where(ok, score_of(lp), -np.inf)
            else:
                if n == NODE_UNCONSTRAINED:
                    cand_tok = np.arange(VL, dtype=np.int64) + vocab_offset
                elif n == NODE_DEAD:
                    cand_tok = np.zeros(0, dtype=np.int64)
                else:
                    ct = csr.children(n)[0].astype(np.int64)
                    if ct.size and (ct.min() < 0 or ct.max() >= V):
                        raise ValueError("CSR child token out of range")
                    cand_tok = ct[(ct >= vocab_offset) & (ct < vocab_offset + VL)]
                lp = lp_of(cand_tok - vocab_offset)
                sc = score_of(lp)

            if eos_token_id >= 0:
                e = np.nonzero(cand_tok == eos_token_id)[0]
                if e.size:
                    out["eos_score"][r, b] = np.float32(sc[e[0]])
                    sc = sc.copy()
                    sc[e] = -np.inf
            flat = b * np.int64(V) + cand_tok
            # the request's top-2B lies within each beam's own top-2B
            keep = topk_canonical(sc, flat, K2)
            pool_s.append(sc[keep])
            pool_f.append(flat[keep])

        if pool_s:
            s = np.concatenate(pool_s)
            f = np.concatenate(pool_f)
        else:
            s = np.zeros(0)
            f = np.zeros(0, np.int64)
        top = topk_canonical(s, f, K2)
        m = top.shape[0]
        out["cand_score64"][r, :m] = s[top]
        out["cand_score"][r, :m] = s[top].astype(np.float32)
        out["cand_token"][r, :m] = (f[top] % V).astype(np.int32)
        out["cand_parent"][r, :m] = (f[top] // V).astype(np.int32)
        mb = min(m, B)
        out["sel_score"][r, :mb] = out["cand_score"][r, :mb]
        out["sel_token"][r, :mb] = out["cand_token"][r, :mb]
        out["sel_parent"][r, :mb] = out["cand_parent"][r, :mb]
        for i in range(mb):
            p = int(out["sel_parent"][r, i])
            t = int(out["sel_token"][r, i])
            out["sel_node"][r, i] = csr.child_of(int(node[r, p]), t) if csr is not None \
                else (NODE_UNCONSTRAINED if node[r, p] == NODE_UNCONSTRAINED else NODE_DEAD)
            if T:
                out["hist_out"][r, i, :T] = hist_in[r, p]
            out["hist_out"][r, i, T] = t
    return out
