"""Data-parallel training step with world_size 2 on CPU (gloo): gradient averaging, replica consistency and
failure detection (a rank that exits makes the peer's collective fail within the process-group timeout)."""
from __future__ import annotations

import os
import socket
import sys
import time
from pathlib import Path

import pytest
import torch
import torch.multiprocessing as mp

ROOT = str(Path(__file__).resolve().parents[1])


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _cfg():
    import sisa_b200 as sisa

    return sisa.SISAConfig(vocab_size=61, d_model=128, n_layer=1, n_head=2, d_ff=64, attn_impl="torch",
                           zero_init_c=False)


def _batch(rank):
    return torch.randint(0, 61, (2, 24), generator=torch.Generator().manual_seed(10 + rank))


def _worker(rank, world, port, mode, q):
    sys.path.insert(0, ROOT)
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world),
                      LOCAL_RANK=str(rank))
    torch.set_num_threads(1)
    from sisa_b200 import dp

    try:
        _, _, dev = dp.init_distributed("gloo", timeout_s=15.0)
        model = dp.build_model(_cfg(), dev, seed=0)
        # SGD: the update is linear in the averaged gradient, so it can be compared with one process
        # the flat form with small buckets (a few parameters each), so several allreduces start during
        # the backward
        trainer = dp.Trainer(model, torch.optim.SGD(model.parameters(), lr=0.5), fused_ce=False,
                             flat_grads=mode in ("flat", "capfail"), bucket_cap_mb=0.05)
        if mode == "flat":
            assert len(trainer._buckets) >= 4, len(trainer._buckets)
        if mode == "exit" and rank == 1:
            os._exit(3)                       # leaves between steps, no collective in flight
        if mode == "capfail":
            _fake_capture(trainer, fail=rank == 1)
        t0 = time.time()
        loss = trainer.step(_batch(rank))
        if mode == "capfail":
            for _ in range(2):                # eager capture attempt and replay steps; all must end eager
                loss = trainer.step(_batch(rank))
            assert not trainer.cuda_graph and trainer._graph is None
        # numpy copies travel by value (tensors would be shared through handles that die with this process)
        q.put((rank, "ok", float(loss), {n: p.detach().numpy().copy() for n, p in model.named_parameters()},
               time.time() - t0))
    except Exception as e:  # noqa: BLE001 - reported to the parent
        q.put((rank, "error", type(e).__name__, str(e)[:200], None))
    finally:
        import torch.distributed as dist

        if dist.is_initialized() and mode != "exit":
            dist.destroy_process_group()


def _fake_capture(trainer, fail):
    """Stand-ins for CUDA-graph capture on CPU: on the failing rank the capture raises; on the other it
    succeeds without running anything (a real capture records kernels but executes none, so it issues
    no collective)."""
    import contextlib
    import warnings

    class _Graph:
        def replay(self):
            raise AssertionError("a graph must not be replayed after a rank failed to capture")

        def reset(self):
            pass

    @contextlib.contextmanager
    def _graph(graph, **kw):
        if fail:
            raise RuntimeError("capture failed (test)")
        real = trainer._forward_backward, trainer._update
        trainer._forward_backward = lambda ids: torch.zeros(())
        trainer._update = lambda: None
        try:
            yield
        finally:
            trainer._forward_backward, trainer._update = real

    warnings.simplefilter("ignore", RuntimeWarning)
    trainer.cuda_graph = True
    torch.cuda.CUDAGraph = _Graph
    torch.cuda.graph = _graph


def _run(mode, world=2, timeout=120):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, mode, q)) for r in range(world)]
    for p in procs:
        p.start()
    out = {}
    expect = 1 if mode == "exit" else world
    t0 = time.time()
    while len(out) < expect and time.time() - t0 < timeout:
        try:
            r = q.get(timeout=5)
            out[r[0]] = r
        except Exception:  # noqa: BLE001 - queue.Empty
            pass
    for p in procs:
        p.join(timeout=30)
        if p.is_alive():
            p.kill()
    return out


@pytest.mark.parametrize("mode", ["ok", "flat"])
def test_dp_gloo_gradients_are_averaged_and_replicas_agree(mode):
    """DDP ("ok") and the flat-gradient form ("flat": one buffer, loss scaled by 1/world, one SUM
    allreduce; the form the multi-GPU CUDA graph captures)."""
    out = _run(mode)
    assert set(out) == {0, 1} and all(v[1] == "ok" for v in out.values()), out
    p0 = {n: torch.from_numpy(a) for n, a in out[0][3].items()}
    p1 = {n: torch.from_numpy(a) for n, a in out[1][3].items()}
    for n in p0:
        assert torch.equal(p0[n], p1[n]), n
    # single process on the concatenated batch gives the same step (equal token counts per rank)
    sys.path.insert(0, ROOT)
    from sisa_b200 import dp

    model = dp.build_model(_cfg(), torch.device("cpu"), seed=0)
    trainer = dp.Trainer(model, torch.optim.SGD(model.parameters(), lr=0.5), fused_ce=False)
    trainer.step(torch.cat([_batch(0), _batch(1)]))
    for n, p in model.named_parameters():
        assert torch.allclose(p.detach(), p0[n], rtol=1e-5, atol=1e-6), n


def test_dp_gloo_capture_failure_on_one_rank_falls_back_everywhere():
    """The graphed data-parallel step captures on every rank, then the ranks agree (MIN of a flag) before
    any replay: if one rank failed to capture, all continue with eager steps of the same form instead
    of one replaying a graph whose allreduce no peer would join."""
    out = _run("capfail")
    assert set(out) == {0, 1} and all(v[1] == "ok" for v in out.values()), out
    for n, a in out[0][3].items():
        assert (a == out[1][3][n]).all(), n


def test_dp_gloo_peer_exit_is_detected():
    out = _run("exit")
    assert 0 in out, out
    rank, status, kind, msg, _ = out[0]
    assert status == "error", out[0]


def test_grad_buckets_start_in_order_once_complete(monkeypatch):
    """Bucket bookkeeping in one process, with the allreduce replaced by a recorder: every bucket starts
    exactly once, in bucket order, and only after each of its parameters has its final gradient."""
    sys.path.insert(0, ROOT)
    from sisa_b200 import dp

    model = dp.build_model(_cfg(), torch.device("cpu"), seed=0)
    params = [p for p in model.parameters() if p.requires_grad]
    starts = []

    def record(view, op=None):
        starts.append((view.data_ptr(), view.numel(), view.clone()))

    monkeypatch.setattr(dp.dist, "all_reduce", record)
    buckets = dp.GradBuckets(params, torch.device("cpu"), cap_mb=0.05)
    assert len(buckets) >= 4
    buckets.start_step()
    loss = model(_batch(0), labels=_batch(0)).loss
    loss.backward()
    buckets.finish()
    assert len(starts) == len(buckets)
    base = buckets.buffer.data_ptr()
    for k, ((ptr, n, snap), (a, b)) in enumerate(zip(starts, buckets.bounds)):
        assert (ptr - base) // 4 == a and n == b - a, k
        assert torch.equal(snap, buckets.buffer[a:b]), f"bucket {k} started before its gradients were final"
    # the gradients are views of the buffer and equal autograd's own
    ref = dp.build_model(_cfg(), torch.device("cpu"), seed=0)
    ref(_batch(0), labels=_batch(0)).loss.backward()
    for (n_, p), q in zip(model.named_parameters(), ref.parameters()):
        assert torch.allclose(p.grad, q.grad, rtol=1e-6, atol=1e-7), n_
    buckets.remove()
