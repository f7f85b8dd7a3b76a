"""Multi-process host logic on CPU (gloo, world size 2): head sharding covers every head once,
timings reduce to the slowest rank, a rank that fails before the collective makes its peer end
with an error instead of hanging, and sharded operator inputs recombine to the full problem
(checked with the oracle)."""
import multiprocessing as mp
import os
import socket
import traceback

import numpy as np
import pytest

from m3ssd import dist as mdist


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, mode, q):
    try:
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank),
                          WORLD_SIZE=str(world))
        import torch.distributed as dist
        mdist.init_process_group("gloo", timeout_s=10.0)
        if mode == "max":
            out = mdist.max_over_ranks([1.0 + rank, 10.0 - rank])
            q.put((rank, "ok", out))
        elif mode == "fail":
            if rank == 1:
                raise RuntimeError("rank 1 failed before the collective")
            try:
                mdist.max_over_ranks([1.0])
                q.put((rank, "no-error", None))
            except Exception as e:  # the collective must error out, not hang
                q.put((rank, "error", type(e).__name__))
        elif mode == "shard":
            from oracle import cases
            from oracle import ssd_oracle as O
            inp, _, chunk = cases.make_case("block_c32")
            import torch
            t = [torch.from_numpy(np.ascontiguousarray(inp[k]))
                 for k in ("x", "A", "B_t", "C_t", "dt")]
            xs = mdist.shard_inputs(*t, world=world, rank=rank)
            y = O.ssd_chunkwise(*[v.numpy() for v in xs], chunk_size=chunk)
            q.put((rank, "ok", (mdist.head_shard(inp["A"].shape[0], world, rank), y)))
        elif mode == "ddp":
            q.put((rank, "ok", _ddp_step(rank)))
        dist.destroy_process_group()
    except Exception as e:
        q.put((rank, "raised", f"{type(e).__name__}: {e}\n{traceback.format_exc()}"))


def _tiny_lm_step(tokens, targets, ddp=False):
    """One train_step of the two-layer model of tests/golden/lm_tiny.npz (CPU SSD restatement,
    fp32) from the fixture's parameters; returns the parameters after the step."""
    import torch
    from m3ssd import lm
    from test_lm_cpu import LM_TINY, _fixture, _ssd_cpu
    _, params, _ = _fixture()
    model = lm.Mamba3Transformer(dict(LM_TINY), ssd_fn=_ssd_cpu)
    model.load_state_dict(params, strict=True)
    net = torch.nn.parallel.DistributedDataParallel(model) if ddp else model
    opt = torch.optim.AdamW(model.parameters(), lr=1e-3)
    lm.train_step(net, opt, tokens, targets, amp_dtype=None)
    return {k: v.detach().numpy().copy() for k, v in model.named_parameters()}


def _ddp_step(rank):
    """Rank r takes row r of the fixture's batch; DDP averages the gradients (complex A
    included), so every rank ends where one process stepping on the whole batch ends."""
    import torch
    from test_lm_cpu import _fixture
    g, _, _ = _fixture()
    tok = torch.from_numpy(g["tokens"][rank:rank + 1])
    tgt = torch.from_numpy(g["targets"][rank:rank + 1])
    return _tiny_lm_step(tok, tgt, ddp=True)


def _run(mode, world=2, timeout=120):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, mode, q)) for r in range(world)]
    for p in procs:
        p.start()
    out = {}
    for _ in range(world):
        r, status, val = q.get(timeout=timeout)
        out[r] = (status, val)
    for p in procs:
        p.join(timeout=60)
        if p.is_alive():
            p.kill()
    return out


@pytest.mark.parametrize("H,world", [(16, 1), (16, 2), (16, 8), (5, 2), (3, 4), (1, 1)])
def test_head_shard_partition(H, world):
    spans = [mdist.head_shard(H, world, r) for r in range(world)]
    covered = [h for a, b in spans for h in range(a, b)]
    assert covered == list(range(H))
    sizes = [b - a for a, b in spans]
    assert max(sizes) - min(sizes) <= 1


def test_head_shard_rejects_bad_rank():
    with pytest.raises(ValueError):
        mdist.head_shard(4, 2, 2)


def test_timings_reduce_to_slowest_rank():
    out = _run("max")
    for r in range(2):
        assert out[r][0] == "ok", out[r]
        assert out[r][1] == [2.0, 10.0]


def test_failed_rank_makes_peer_error_not_hang():
    out = _run("fail", timeout=180)
    assert out[1][0] == "raised"
    assert out[0][0] == "error", out[0]


def test_sharded_problem_recombines():
    from oracle import cases
    from oracle import ssd_oracle as O
    out = _run("shard")
    inp, _, chunk = cases.make_case("block_c32")
    y_full = O.ssd_chunkwise(**inp, chunk_size=chunk)
    for r in range(2):
        assert out[r][0] == "ok", out[r]
        (h0, h1), y = out[r][1]
        np.testing.assert_array_equal(y, y_full[:, :, h0:h1])


def test_ddp_train_step_matches_one_process_on_the_whole_batch():
    """The whole-model data-parallel step (m3ssd.lm under DistributedDataParallel, gloo, two
    ranks, one row of the batch each) ends with the parameters one process reaches on both rows."""
    import torch
    from test_lm_cpu import _fixture
    out = _run("ddp", timeout=300)
    g, _, _ = _fixture()
    want = _tiny_lm_step(torch.from_numpy(g["tokens"]), torch.from_numpy(g["targets"]))
    for r in range(2):
        assert out[r][0] == "ok", out[r]
        got = out[r][1]
        assert sorted(got) == sorted(want)
        for k in want:
            np.testing.assert_allclose(got[k], want[k], rtol=2e-5, atol=2e-6, err_msg=k)
