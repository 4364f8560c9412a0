"""Run the reference's own beam-search loops on a mock engine (TEST INFRASTRUCTURE).

Used only by tests/golden/make_golden.py to record golden vectors from the
reference implementation itself.  Nothing in the package imports it, and it
needs the reference checkout (its path is passed in; it is not available on
GPU boxes, which only read the committed fixtures).

The reference pins vLLM 0.14; the installed vLLM is newer and moved a few
modules the reference imports.  ``install()`` registers stand-ins for exactly
those names (everything else resolves to the installed vLLM):

  vllm.beam_search            BeamSearchSequence / BeamSearchInstance /
                              BeamSearchOutput dataclasses and
                              create_sort_beams_key_function (vLLM's published
                              length-penalised sort key)
  vllm.inputs.data            PromptType, TokensPrompt
  vllm.inputs.parse           is_explicit_encoder_decoder_prompt (always False)
  vllm.entrypoints.openai.protocol        VLLMValidationError
  vllm.entrypoints.openai.serving_models  BaseModelPath, LoRAModulePath,
                                          OpenAIServingModels (empty stand-ins)
  vllm.multimodal.MultiModalDataDict

The mock engine restates vLLM's sampler for a beam: float32 logits of the
beam's full token sequence (content addressed, so the reference's unordered
beam order cannot change its inputs; optionally rounded to bf16 values, as a
bf16 model's logits are), lp = log_softmax(logits) -- or, with vLLM's
logprobs_mode "processed_logprobs", log_softmax(logits / T) with the
temperature the reference's loop put in its SamplingParams (T < 1e-5 counts
as 1) -- and the top-K list [sampled, top1..topK] with the greedy token as
`sampled` (vllm v1/sample/sampler.py:223-233, 300-352).  In "allowed" mode the top-K list holds
the beam's best K catalog children (so the reference's own mask/add/EOS/select
code yields the constrained result); in "raw" mode it is the plain top-K and the
reference masks it itself (serving_engine.py:504-506).
"""
from __future__ import annotations

import asyncio
import dataclasses
import hashlib
import sys
import types
from typing import Any, Callable

import numpy as np


# ---------------------------------------------------------------- stand-ins
@dataclasses.dataclass
class BeamSearchSequence:
    tokens: list
    logprobs: Any
    lora_request: Any = None
    cum_logprob: float = 0.0
    text: str | None = None
    finish_reason: str | None = None
    stop_reason: Any = None
    multi_modal_data: Any = None
    mm_processor_kwargs: Any = None


@dataclasses.dataclass
class BeamSearchOutput:
    sequences: list


class BeamSearchInstance:
    def __init__(self, prompt_tokens, lora_request=None, logprobs=None, **kwargs):
        self.beams = [BeamSearchSequence(tokens=list(prompt_tokens), logprobs=[] if logprobs is None else list(logprobs),
                                         lora_request=lora_request, **kwargs)]
        self.completed = []


def create_sort_beams_key_function(eos_token_id, length_penalty):
    """vLLM's beam score: cum_logprob / len**length_penalty, the EOS token not counted."""
    def key(x):
        seq_len = len(x.tokens)
        if x.tokens and x.tokens[-1] == eos_token_id:
            seq_len -= 1
        return x.cum_logprob / (seq_len ** length_penalty)
    return key


class VLLMValidationError(ValueError):
    def __init__(self, message, parameter=None, value=None):
        super().__init__(message)
        self.parameter = parameter
        self.value = value


def install(reference_root: str) -> None:
    """Put the reference on sys.path and register the missing vLLM names."""
    if reference_root not in sys.path:
        sys.path.insert(0, reference_root)
    import vllm.inputs as vinputs

    def mod(name, **attrs):
        m = types.ModuleType(name)
        for k, v in attrs.items():
            setattr(m, k, v)
        sys.modules[name] = m
        return m

    mod("vllm.beam_search", BeamSearchSequence=BeamSearchSequence, BeamSearchInstance=BeamSearchInstance,
        BeamSearchOutput=BeamSearchOutput, create_sort_beams_key_function=create_sort_beams_key_function)
    mod("vllm.inputs.data", PromptType=Any, TokensPrompt=vinputs.TokensPrompt, TextPrompt=vinputs.TextPrompt)
    mod("vllm.inputs.parse", is_explicit_encoder_decoder_prompt=lambda p: False)
    import vllm.entrypoints.openai as voa

    class _ServingModels:
        def __init__(self, *a, **k):
            pass

    mod("vllm.entrypoints.openai.protocol", VLLMValidationError=VLLMValidationError)
    mod("vllm.entrypoints.openai.serving_models", BaseModelPath=object, LoRAModulePath=object,
        OpenAIServingModels=_ServingModels)
    voa.protocol = sys.modules["vllm.entrypoints.openai.protocol"]
    voa.serving_models = sys.modules["vllm.entrypoints.openai.serving_models"]
    import vllm.multimodal as vmm
    if not hasattr(vmm, "MultiModalDataDict"):
        vmm.MultiModalDataDict = dict


def install_attention(reference_root: str) -> None:
    """Make the reference's beam attention backend importable on a CPU-only
    host with the installed vLLM: stand-ins for the four names it imports that
    this vLLM does not have (is_quantized_kv_cache, flash_attn_supports_fp8,
    vllm_is_batch_invariant: constant False; AttentionMetadataBuilder: an empty
    generic base).  Only its metadata builder (plain Python) is used."""
    install(reference_root)
    import typing
    import vllm.model_executor.layers.batch_invariant as bi
    import vllm.v1.attention.backend as vb
    import vllm.v1.attention.backends.fa_utils as fu
    import vllm.v1.attention.backends.utils as vu
    if not hasattr(vb, "is_quantized_kv_cache"):
        vb.is_quantized_kv_cache = lambda *a, **k: False
    if not hasattr(fu, "flash_attn_supports_fp8"):
        fu.flash_attn_supports_fp8 = lambda *a, **k: False
    if not hasattr(bi, "vllm_is_batch_invariant"):
        bi.vllm_is_batch_invariant = lambda *a, **k: False
    if not hasattr(vu, "AttentionMetadataBuilder"):
        T = typing.TypeVar("T")

        class AttentionMetadataBuilder(typing.Generic[T]):
            pass

        vu.AttentionMetadataBuilder = AttentionMetadataBuilder


def reference_suffix_metadata(reference_root: str, *, num_reqs, beam_width, q_seq_len, prefix_len, steps,
                              cache_len, block_size, block_tables, slot_mapping):
    """Run the reference's BeamAttentionMetadataBuilder.build (beam_attn.py:480-559)
    for mega-decode requests laid out as in its own kernel test
    (tests/kernels/attention/test_cascade_beam_flash_attn.py:322-380) and return
    the suffix-pass metadata it builds."""
    install_attention(reference_root)
    import torch
    from vllm_gr.v1.attention.backends.beam_attn import MEGA_DATA_VAR, BeamAttentionMetadataBuilder

    class Common:
        pass

    cm = Common()
    cm.num_reqs = num_reqs
    cm.query_start_loc_cpu = torch.arange(0, (num_reqs * beam_width + 1) * q_seq_len, beam_width * q_seq_len,
                                          dtype=torch.int32)
    cm.query_start_loc = cm.query_start_loc_cpu
    cm.seq_lens = torch.full((num_reqs,), prefix_len + beam_width * steps, dtype=torch.int32)
    cm.block_table_tensor = block_tables
    cm.num_actual_tokens = num_reqs * beam_width * q_seq_len
    cm.max_query_len = q_seq_len * beam_width
    cm.max_seq_len = prefix_len + beam_width * steps
    cm.causal = True
    cm.slot_mapping = slot_mapping
    info = {"mega_data": {f"req_{i}": {"is_mega_decode": True, "prefix_len": prefix_len,
                                       "mega_beam_width": beam_width, "mega_decode_steps": steps,
                                       "cache_len": cache_len} for i in range(num_reqs)},
            "req_ids": [f"req_{i}" for i in range(num_reqs)]}
    token = MEGA_DATA_VAR.set(info)
    try:
        b = BeamAttentionMetadataBuilder.__new__(BeamAttentionMetadataBuilder)
        b.device = "cpu"
        b.block_size = block_size
        b.aot_schedule = False
        b.aot_sliding_window = None
        b.use_full_cuda_graph = False
        b.max_cudagraph_size = None
        b.max_num_splits = 0
        m = b.build(common_prefix_len=prefix_len, common_attn_metadata=cm, fast_build=False)
    finally:
        MEGA_DATA_VAR.reset(token)

    def lst(x):
        return None if x is None else x.tolist()

    return {
        "mega_prefix_indices": lst(m.mega_prefix_indices),
        "suffix_slot_mapping_out": lst(m.mega_suffix_slot_mapping_out),
        "suffix_total_tokens": int(m.mega_suffix_total_tokens),
        "suffix_seq_lens": lst(m.mega_suffix_seq_lens),
        "suffix_cu_seqlens_q": lst(m.mega_suffix_cu_seqlens_q),
        "suffix_cu_seqlens_k": lst(m.mega_suffix_cu_seqlens_k),
    }


# ---------------------------------------------------------------- mock sampler
def beam_logits(tokens, vocab: int, sigma: float, seed: int, bf16: bool) -> np.ndarray:
    """float32 logits of one beam, a function of its whole token sequence."""
    h = hashlib.sha256((str(seed) + ":" + ",".join(map(str, tokens))).encode()).digest()
    rng = np.random.default_rng(int.from_bytes(h[:8], "little"))
    x = (rng.standard_normal(vocab, dtype=np.float32) * np.float32(sigma)).astype(np.float32)
    if bf16:
        u = x.view(np.uint32).astype(np.uint64)
        u = ((u + (((u >> 16) & 1) + 0x7FFF)) >> 16) << 16
        x = u.astype(np.uint32).view(np.float32)
    return x


def log_softmax32(x: np.ndarray) -> np.ndarray:
    import torch
    return torch.log_softmax(torch.from_numpy(x), dim=-1).numpy()


def top_list(lp: np.ndarray, k: int, allowed: np.ndarray | None):
    """Token ids of the top-k log-probs (ties: lower id first); with `allowed`,
    the best allowed ids first, padded by the best disallowed ones."""
    ids = np.lexsort((np.arange(lp.shape[0]), -lp.astype(np.float64)))
    if allowed is None:
        return ids[:k]
    mask = np.zeros(lp.shape[0], bool)
    mask[allowed] = True
    good = ids[mask[ids]]
    bad = ids[~mask[ids]]
    return np.concatenate([good, bad])[:k]


class MockEngine:
    """Engine client for serving_engine.beam_search (ADD_BATCH path) and an LLM
    stand-in for llm.beam_search: every request is one beam advancing one token."""

    def __init__(self, vocab, sigma, seed, bf16, prompt_len_of: Callable | None = None, allowed_fn=None,
                 processed: bool = False):
        self.vocab, self.sigma, self.seed, self.bf16 = vocab, sigma, seed, bf16
        self.processed = processed            # vLLM logprobs_mode "processed_logprobs"
        self.allowed_fn = allowed_fn          # tokens -> allowed child ids (or None = raw top-K)
        self.calls: list[list[list[int]]] = []  # beams requested per step
        self._pending: dict = {}

    def output_for(self, tokens, k, temperature=None):
        from vllm.logprobs import FlatLogprobs
        from vllm.outputs import CompletionOutput
        x = beam_logits(tokens, self.vocab, self.sigma, self.seed, self.bf16)
        if self.processed and temperature is not None and temperature >= 1e-5:
            x = (x / np.float32(temperature)).astype(np.float32)
        lp = log_softmax32(x)
        allowed = None if self.allowed_fn is None else self.allowed_fn(tokens)
        top = top_list(lp, k, allowed)
        sampled = int(top[0])
        ids = [sampled] + [int(t) for t in top]
        flat = FlatLogprobs()
        flat.start_indices.append(0)
        flat.token_ids.extend(ids)
        flat.logprobs.extend(float(lp[t]) for t in ids)
        flat.ranks.extend([None] * len(ids))
        flat.decoded_tokens.extend([None] * len(ids))
        flat.end_indices.append(len(ids))
        return CompletionOutput(index=0, text="", token_ids=[sampled], cumulative_logprob=None, logprobs=flat,
                                finish_reason="length")

    # ---- engine client (online) ----
    def prepare_request(self, request_id, prompt, params, **kwargs):
        q = asyncio.Queue()
        req = types.SimpleNamespace(request_id=request_id, tokens=list(prompt["prompt_token_ids"]),
                                    k=params.logprobs, temperature=params.temperature, queue=q, metrics=None)
        return q, req

    async def _add_requests_batch(self, reqs, use_batch_message=False):
        self.calls.append([list(r.tokens) for r in reqs])
        for r in reqs:
            out = types.SimpleNamespace(outputs=[self.output_for(r.tokens, r.k, r.temperature)], finished=True,
                                        metrics=None)
            await r.queue.put(out)

    # ---- LLM stand-in (offline) ----
    def generate(self, prompts, sampling_params=None, use_tqdm=False, lora_request=None):
        self.calls.append([list(p["prompt_token_ids"]) for p in prompts])
        return [types.SimpleNamespace(outputs=[self.output_for(list(p["prompt_token_ids"]), sampling_params.logprobs,
                                                               sampling_params.temperature)])
                for p in prompts]


class Tok:
    """Tokenizer stand-in: token strings are decimal ids."""

    def __init__(self, eos_token_id):
        self.eos_token_id = eos_token_id

    def convert_tokens_to_ids(self, t):
        if isinstance(t, list):
            return [int(x) for x in t]
        return int(t)

    def encode(self, s):
        return [int(x) for x in s.split()]

    def decode(self, tokens):
        return " ".join(map(str, tokens))


def run_online(reference_root, prompt_tokens, *, beam_width, max_tokens, vocab, sigma, seed, bf16, catalog_seqs,
               begin_token, end_token, eos_token_id, ignore_eos, mode, processed=False, temperature=0.0):
    """serving_engine.beam_search with a catalog; returns (calls, final beams)."""
    install(reference_root)
    from vllm_gr.entrypoints.openai import serving_engine
    from vllm_gr.entrypoints.openai.serving_models import Catalog
    from vllm_gr.sampling_params import BeamSearchParams

    tok = Tok(eos_token_id)
    cat = Catalog(tok)
    cat.trie = {}
    for seq in catalog_seqs:                         # Catalog.load's loop, without the JSON file
        node = cat.trie
        for t in seq:
            node = node.setdefault(int(t), {})
    plen = len(prompt_tokens)
    allowed_fn = None
    if mode == "allowed":
        allowed_fn = lambda toks: np.array(sorted(cat.valid(toks[plen:])), dtype=np.int64)  # noqa: E731
    eng = MockEngine(vocab, sigma, seed, bf16, allowed_fn=allowed_fn, processed=processed)
    this = types.SimpleNamespace(engine_client=eng, input_processor=types.SimpleNamespace(tokenizer=tok),
                                 models=types.SimpleNamespace(catalog=cat))
    params = BeamSearchParams(beam_width=beam_width, max_tokens=max_tokens, ignore_eos=ignore_eos,
                              temperature=temperature,
                              begin_token=None if begin_token is None else str(begin_token),
                              end_token=None if end_token is None else str(end_token))

    async def go():
        res = None
        async for out in serving_engine.beam_search(this, {"prompt_token_ids": list(prompt_tokens)}, "req", params):
            res = out
        return res

    out = asyncio.run(go())
    beams = [(list(o.token_ids), float(o.cumulative_logprob), o.finish_reason) for o in out.outputs]
    return eng.calls, beams


def run_offline(reference_root, prompts, *, beam_width, max_tokens, vocab, sigma, seed, bf16, eos_token_id,
                ignore_eos, length_penalty, processed=False, temperature=0.0):
    """llm.beam_search (no catalog); returns (calls, final beams per prompt)."""
    install(reference_root)
    from vllm_gr.entrypoints import llm as llm_mod
    from vllm_gr.sampling_params import BeamSearchParams

    tok = Tok(eos_token_id)
    eng = MockEngine(vocab, sigma, seed, bf16, processed=processed)
    this = types.SimpleNamespace(_get_beam_search_lora_requests=lambda lr, ps: [None] * len(ps),
                                 get_tokenizer=lambda: tok, generate=eng.generate)
    params = BeamSearchParams(beam_width=beam_width, max_tokens=max_tokens, ignore_eos=ignore_eos,
                              temperature=temperature, length_penalty=length_penalty)
    outs = llm_mod.beam_search(this, [{"prompt_token_ids": list(p)} for p in prompts], params)
    return eng.calls, [[(list(s.tokens), float(s.cum_logprob), s.finish_reason) for s in o.sequences] for o in outs]
