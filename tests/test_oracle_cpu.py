"""Oracle properties on the CPU (the oracle is pinned to the reference's own
loops by tests/test_golden_reference.py; these cover the parts the golden
cases do not reach)."""
import numpy as np
import torch

from oracle import restated as O


def test_penalties_follow_vllm_apply_penalties():
    # independent restatement with vLLM's tensor operations (model_executor/layers/utils.py:51-89;
    # repetition as the CUDA op: x > 0 ? x / p : x * p), float32 throughout
    rng = np.random.default_rng(0)
    V = 300
    x = (rng.standard_normal(V) * 3).astype(np.float32)
    hist = rng.integers(0, V, 40).astype(np.int32)
    rep, pres, freq = 1.3, 0.4, 0.2
    t = torch.from_numpy(x.copy())[None]
    counts = torch.zeros((1, V + 1), dtype=torch.long)
    counts.scatter_add_(1, torch.from_numpy(hist.astype(np.int64))[None], torch.ones((1, hist.shape[0]), dtype=torch.long))
    counts = counts[:, :V]
    mask = counts > 0
    t = torch.where(mask & (t > 0), t / rep, torch.where(mask, t * rep, t))
    t = t - torch.tensor([freq], dtype=torch.float32)[:, None] * counts
    t = t - torch.tensor([pres], dtype=torch.float32)[:, None] * mask
    got = O.penalise_row(x, hist, 0, rep, pres, freq)
    assert np.array_equal(got.view(np.uint32), t[0].numpy().view(np.uint32))


def test_temperature_and_greedy_eps():
    x = np.array([1.0, -2.0, 3.5], np.float32)
    assert np.array_equal(O.processed_row(x, None, 0, 0.7, 1.0, 0.0, 0.0), (x / np.float32(0.7)).astype(np.float32))
    assert np.array_equal(O.processed_row(x, None, 0, 0.0, 1.0, 0.0, 0.0), x)     # T < 1e-5 -> 1


def test_canonical_ties_lowest_flat_index_first():
    R, NB, V, B = 1, 3, 16, 4
    x = np.zeros((R, NB, V), np.float32)
    out = O.beam_step(x, np.zeros((R, NB), np.float32), np.full((R, NB), -1, np.int32), None, beam_width=B,
                      vocab_size=V)
    # all scores equal: parent 0 tokens 0..7 first
    assert out["cand_parent"][0].tolist() == [0] * 8
    assert out["cand_token"][0].tolist() == list(range(8))


def test_eos_recorded_and_removed_from_pool():
    R, NB, V, B = 1, 2, 8, 2
    x = np.full((R, NB, V), -5.0, np.float32)
    x[0, 0, 3] = 5.0             # EOS is beam 0's best token
    out = O.beam_step(x, np.array([[0.0, -1.0]], np.float32), np.full((R, NB), -1, np.int32), None,
                      beam_width=B, vocab_size=V, eos_token_id=3)
    assert np.isfinite(out["eos_score"][0]).all()
    assert 3 not in out["sel_token"][0].tolist()


def test_literal_mode_sampled_token_dedup():
    # raw log-probs, penalties push the greedy token outside the raw top-K: it replaces the K-th entry
    V, K = 32, 3
    x = np.linspace(0, 3, V, dtype=np.float32)[None, None, :]   # best raw tokens: 31, 30, 29
    hist = np.array([[[31, 30, 29]]], np.int32)
    out = O.beam_step(x, np.zeros((1, 1), np.float32), np.full((1, 1), -1, np.int32), None, beam_width=2,
                      vocab_size=V, per_beam_k=K, hist_in=hist, rep_penalty=[10.0], pres_penalty=[5.0])
    # greedy over penalised logits is token 28, not in the raw top-3 -> candidates {28, 31, 30}
    assert sorted(out["cand_token"][0][:3].tolist()) == [28, 30, 31]


def test_device_and_reference_arithmetic_agree_on_random_case():
    rng = np.random.default_rng(5)
    R, NB, V, B = 2, 6, 500, 6
    x = (rng.standard_normal((R, NB, V)) * 3).astype(np.float32)
    cum = np.sort(rng.uniform(-10, 0, (R, NB)).astype(np.float32))[:, ::-1].copy()
    node = np.full((R, NB), -1, np.int32)
    a = O.beam_step(x, cum, node, None, beam_width=B, vocab_size=V, arith="reference")
    b = O.beam_step(x, cum, node, None, beam_width=B, vocab_size=V, arith="device")
    assert np.array_equal(a["cand_token"], b["cand_token"]) and np.array_equal(a["cand_parent"], b["cand_parent"])
    assert np.allclose(a["cand_score"], b["cand_score"], rtol=1e-6)


def test_fork_table():
    R, NB, V, B = 1, 2, 10, 2
    x = np.full((R, NB, V), -5.0, np.float32)
    x[0, 1, 7] = 4.0
    x[0, 0, 2] = 3.0
    hist = np.array([[[1, 2], [3, 4]]], np.int32)
    out = O.beam_step(x, np.zeros((R, NB), np.float32), np.full((R, NB), -1, np.int32), None, beam_width=B,
                      vocab_size=V, hist_in=hist)
    assert out["hist_out"][0].tolist() == [[3, 4, 7], [1, 2, 2]]
