"""Vocab-sharded step across real GPUs: one process per GPU, NCCL all-gathers
(torch_all_gather), each rank holding a contiguous column slice of the logits,
then the strided split (rank k: tokens k, k + 2, ...).  Every rank's outputs
must equal the oracle's full-vocabulary step (bit-exact given the combined
lse).  Needs two GPUs; skipped otherwise."""
import os
import socket

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, q):
    try:
        import datetime
        import sys
        import torch
        import torch.distributed as dist
        sys.path.insert(0, os.path.dirname(__file__))
        from helpers import Case, make_logits, small_catalog, to_device_logits, OUT_KEYS
        from vllm_gr_ehaleva_b200.sharded import sharded_beam_step, torch_all_gather
        from vllm_gr_ehaleva_b200.synthetic import initial_cum
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
        torch.cuda.set_device(rank)
        dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
        cat = small_catalog()
        R, NB, B, V = 2, 16, 16, 8192
        case = Case(logits32=make_logits(R, NB, V, 4.0, 21, "bf16"), dtype="bf16", cum=initial_cum(R, NB),
                    node=np.full((R, NB), cat.start_node, np.int32), beam_width=B, vocab_size=V, csr=cat.csr,
                    hist=np.full((R, NB, 1), cat.sid_begin, np.int32))
        dev = torch.device("cuda", rank)
        VL = V // world
        full = to_device_logits(case, dev)
        csr = tuple(torch.from_numpy(a).to(dev) for a in (cat.csr.row_ptr, cat.csr.child_tok, cat.csr.child_node))
        from vllm_gr_ehaleva_b200.sharded import ShardedStepper
        results = {}
        for split in ("contiguous", "strided"):
            if split == "strided":
                local, voff, vs = full[:, rank::world].contiguous(), rank, world
            else:
                local, voff, vs = full[:, rank * VL:(rank + 1) * VL], rank * VL, 1
            out = sharded_beam_step(local, torch.from_numpy(case.cum).to(dev), torch.from_numpy(case.node).to(dev),
                                    all_gather=torch_all_gather(), beam_width=B, vocab_size=V, vocab_offset=voff,
                                    vocab_stride=vs, csr=csr, hist=torch.from_numpy(case.hist).to(dev))
            torch.cuda.synchronize()
            res = {k: getattr(out, k).cpu().numpy() for k in OUT_KEYS}
            res["err"] = int(out.err.item())
            # the persistent stepper gives the same step
            stepper = ShardedStepper(num_requests=R, num_beams=NB, beam_width=B, vocab_size=V, vocab_local=VL,
                                     vocab_offset=voff, vocab_stride=vs, num_shards=world, csr=csr, hist_len=1,
                                     row_stride=local.stride(0), device=dev)
            out2 = stepper.step(local, torch.from_numpy(case.cum).to(dev), torch.from_numpy(case.node).to(dev),
                                torch.from_numpy(case.hist).to(dev))
            torch.cuda.synchronize()
            res["stepper_same"] = all(np.array_equal(getattr(out2, k).cpu().numpy(), res[k])
                                      for k in ("cand_score", "cand_token", "cand_parent", "sel_node", "hist_out"))
            results[split] = res
        q.put((rank, results))
        dist.barrier()
        dist.destroy_process_group()
    except Exception as e:
        q.put((rank, {"error": repr(e)}))


def test_sharded_step_two_gpus_nccl():
    import torch
    import torch.multiprocessing as mp
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    from helpers import Case, assert_step_parity, make_logits, small_catalog
    from vllm_gr_ehaleva_b200.synthetic import initial_cum
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    results = dict(q.get(timeout=300) for _ in procs)
    for p in procs:
        p.join(timeout=120)
    cat = small_catalog()
    R, NB, B, V = 2, 16, 16, 8192
    case = Case(logits32=make_logits(R, NB, V, 4.0, 21, "bf16"), dtype="bf16", cum=initial_cum(R, NB),
                node=np.full((R, NB), cat.start_node, np.int32), beam_width=B, vocab_size=V, csr=cat.csr,
                hist=np.full((R, NB, 1), cat.sid_begin, np.int32))
    for r in range(2):
        assert "error" not in results[r], results[r]
    for split in ("contiguous", "strided"):
        for r in range(2):
            res = results[r][split]
            assert res.pop("stepper_same"), split
            assert_step_parity(case, res, label=f"nccl {split} rank {r}")
        for k in ("cand_token", "cand_parent", "sel_node", "hist_out"):
            assert np.array_equal(results[0][split][k], results[1][split][k]), (split, k)
