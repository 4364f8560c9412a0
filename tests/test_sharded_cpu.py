"""Host orchestration of the vocab-sharded step on two gloo ranks (CPU).

The three device phases are replaced by stand-ins that tag their outputs with
the rank, so the test checks what the orchestration moves between them: the
partials and keys all-gathered in rank order, the merge fed every rank's keys,
the EOS score taken from the rank that owns it, and the error words OR-ed."""
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

R, NB, B = 2, 3, 2


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, result_q):
    try:
        os.environ["MASTER_ADDR"] = "127.0.0.1"
        os.environ["MASTER_PORT"] = str(port)
        dist.init_process_group("gloo", rank=rank, world_size=world)
        from vllm_gr_ehaleva_b200 import sharded as SH
        from vllm_gr_ehaleva_b200.sample.beam_search_sampler import BeamStepOutput

        seen = {}

        def fake_partials(local, cum, node, **kw):
            assert kw["vocab_offset"] == rank * 10 and kw["per_beam_k"] == 0
            t = torch.full((R * NB, 2), float(rank))
            t.err = torch.tensor([1 << rank], dtype=torch.int32)
            return t

        def fake_shard(local, cum, node, gathered, **kw):
            seen["partials"] = gathered.clone()
            keys = torch.full((R, 2 * B), 100 + rank, dtype=torch.int64)
            lse = torch.full((R, NB), 7.0)
            eos = torch.full((R, NB), float("nan"))
            if rank == 1:                         # the rank whose columns hold EOS
                eos[0, 1] = -3.5
            return keys, lse, eos, torch.tensor([1 << (2 + rank)], dtype=torch.int32)

        def fake_merge(local, cum, node, gathered_keys, **kw):
            seen["keys"] = gathered_keys.clone()
            z = torch.zeros
            return BeamStepOutput(cand_score=z(R, 2 * B), cand_token=z(R, 2 * B, dtype=torch.int32),
                                  cand_parent=z(R, 2 * B, dtype=torch.int32), sel_score=z(R, B),
                                  sel_token=z(R, B, dtype=torch.int32), sel_parent=z(R, B, dtype=torch.int32),
                                  sel_node=z(R, B, dtype=torch.int32), eos_score=z(R, NB),
                                  hist_out=z(R, B, 1, dtype=torch.int32), lse=z(R, NB),
                                  err=torch.tensor([1 << (4 + rank)], dtype=torch.int32))

        SH.lse_partials, SH.shard_candidates, SH.merge_candidates = fake_partials, fake_shard, fake_merge
        out = SH.sharded_beam_step(torch.zeros(R * NB, 10), torch.zeros(R, NB), torch.zeros(R, NB, dtype=torch.int32),
                                   all_gather=SH.torch_all_gather(), beam_width=B, vocab_size=10 * world,
                                   vocab_offset=rank * 10, eos_token_id=13)
        res = {
            "partials_order": [float(seen["partials"][k, 0, 0]) for k in range(world)],
            "keys_order": [int(seen["keys"][k, 0, 0]) for k in range(world)],
            "eos": out.eos_score.tolist(),
            "lse": float(out.lse[0, 0]),
            "err": int(out.err.item()),
        }
        result_q.put((rank, res))
        dist.barrier()
        dist.destroy_process_group()
    except Exception as e:                       # report to the parent instead of hanging it
        result_q.put((rank, {"error": repr(e)}))


def test_sharded_orchestration_two_gloo_ranks():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    results = dict(q.get(timeout=120) for _ in procs)
    for p in procs:
        p.join(timeout=60)
    for r in range(2):
        res = results[r]
        assert "error" not in res, res
        assert res["partials_order"] == [0.0, 1.0]          # rank order
        assert res["keys_order"] == [100, 101]
        assert res["lse"] == 7.0
        assert res["eos"][0][1] == -3.5                     # from the owning rank
        assert all(v != v for i, row in enumerate(res["eos"]) for j, v in enumerate(row) if (i, j) != (0, 1))
        # this rank's three calls' error words, OR-ed
        assert res["err"] == (1 << r) | (1 << (2 + r)) | (1 << (4 + r))


def _dropout_worker(rank, world, port, result_q):
    # rank 1 leaves before the step; rank 0's first all-gather must fail, not hang
    import datetime
    import time
    try:
        os.environ["MASTER_ADDR"] = "127.0.0.1"
        os.environ["MASTER_PORT"] = str(port)
        dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=5))
        if rank == 1:
            result_q.put((rank, {"left": True}))
            result_q.close()
            result_q.join_thread()                # the message is out before the process is
            os._exit(0)                           # no barrier, no destroy: a rank that drops out
        from vllm_gr_ehaleva_b200 import sharded as SH

        def fake_partials(local, cum, node, **kw):
            t = torch.zeros((R * NB, 2))
            t.err = torch.zeros(1, dtype=torch.int32)
            return t

        SH.lse_partials = fake_partials
        t0 = time.monotonic()
        try:
            SH.sharded_beam_step(torch.zeros(R * NB, 10), torch.zeros(R, NB), torch.zeros(R, NB, dtype=torch.int32),
                                 all_gather=SH.torch_all_gather(), beam_width=B, vocab_size=20, vocab_offset=0,
                                 eos_token_id=13)
            result_q.put((rank, {"raised": False}))
        except Exception as e:                    # the collective's error surfaces to the caller
            result_q.put((rank, {"raised": True, "kind": type(e).__name__, "secs": time.monotonic() - t0}))
    except Exception as e:
        result_q.put((rank, {"error": repr(e)}))


def test_rank_dropout_surfaces_as_an_error():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_dropout_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    results = dict(q.get(timeout=120) for _ in procs)
    for p in procs:
        p.join(timeout=60)
        if p.is_alive():
            p.kill()
    assert results[1] == {"left": True}
    assert "error" not in results[0], results[0]
    assert results[0]["raised"] and results[0]["secs"] < 60, results[0]
