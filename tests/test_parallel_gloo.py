"""World-size-2 data-parallel host logic on CPU (gloo): batch sharding plus the single
gradient all-reduce reproduce the one-process full-batch gradients, and a rank that dies
before the collective makes its peer fail instead of hanging."""
import os
import socket
import sys

import pytest
import torch
import torch.multiprocessing as mp

HERE = os.path.dirname(os.path.abspath(__file__))


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _use_cpu_prologue(setattr_fn=setattr):
    import ttc_b200.layer as L
    from prologue_ref import _l2norm, prologue_torch
    setattr_fn(L, "prologue", prologue_torch)  # CPU stand-in for the CUDA prologue
    setattr_fn(L, "rownorm", _l2norm)          # and for the CUDA epilogue


def _layer():
    from oracle import ttc_oracle as O
    from ttc_b200 import TTCLayer
    torch.manual_seed(0)
    layer = TTCLayer(8, 6, 16, 2, 16, 16).double()
    layer.solver = O.fused_solve          # CPU stand-in for the CUDA solver
    return layer


def _data():
    g = torch.Generator().manual_seed(5)
    return torch.randn(4, 6, 8, generator=g, dtype=torch.float64), \
        torch.randn(4, 6, 6, generator=g, dtype=torch.float64)


def _worker(rank, world, port, out_dir, fail_rank, overlapped=False):
    for p in (os.path.dirname(HERE), os.path.join(os.path.dirname(HERE), "ttc-net_b200"), HERE):
        sys.path.insert(0, p)
    import datetime

    import torch.distributed as dist
    from ttc_b200.parallel import allreduce_grads, shard_rows
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=20))
    _use_cpu_prologue()
    layer = _layer()
    x, dy = _data()
    xs, dys = shard_rows(x, rank, world), shard_rows(dy, rank, world)
    if overlapped:
        # micro-batches of 5 rows, each gradient all-reduced as soon as the last one has
        # completed it (the bench's N > 1 step)
        from ttc_b200.parallel import OverlappedGradAllReduce
        red = OverlappedGradAllReduce(layer)
        layer.forward_backward(xs, dys, 5, rows=5, before_last_backward=red.arm)
        red.wait()
        torch.save({n: p.grad for n, p in layer.named_parameters()},
                   os.path.join(out_dir, f"grads{rank}.pt"))
        dist.destroy_process_group()
        return
    y = layer(xs, T=5)
    y.backward(dys)
    if rank == fail_rank:
        os._exit(3)                      # dies between steps, no collective in flight
    allreduce_grads(layer)
    torch.save({n: p.grad for n, p in layer.named_parameters()},
               os.path.join(out_dir, f"grads{rank}.pt"))
    dist.destroy_process_group()


def _run(world, tmp_path, fail_rank=-1, overlapped=False):
    ctx = mp.get_context("spawn")
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, str(tmp_path), fail_rank, overlapped))
             for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
    alive = [p for p in procs if p.is_alive()]
    for p in alive:
        p.kill()
    assert not alive, "a rank hung"
    return [p.exitcode for p in procs]


def test_sharded_gradients_equal_full_batch(tmp_path, monkeypatch):
    _use_cpu_prologue(monkeypatch.setattr)
    codes = _run(2, tmp_path)
    assert codes == [0, 0]
    layer = _layer()
    x, dy = _data()
    layer(x, T=5).backward(dy)
    for r in range(2):
        g = torch.load(os.path.join(tmp_path, f"grads{r}.pt"))
        for n, p in layer.named_parameters():
            assert torch.allclose(g[n], p.grad, rtol=1e-10, atol=1e-12), n


def test_overlapped_allreduce_of_micro_batches_equals_full_batch(tmp_path, monkeypatch):
    """forward_backward over micro-batches with each parameter's all-reduce started from its
    post-accumulate hook gives every rank the full-batch gradients."""
    _use_cpu_prologue(monkeypatch.setattr)
    codes = _run(2, tmp_path, overlapped=True)
    assert codes == [0, 0]
    layer = _layer()
    x, dy = _data()
    layer(x, T=5).backward(dy)
    for r in range(2):
        g = torch.load(os.path.join(tmp_path, f"grads{r}.pt"))
        for n, p in layer.named_parameters():
            assert torch.allclose(g[n], p.grad, rtol=1e-10, atol=1e-12), n


def test_rank_failure_is_reported_not_hung(tmp_path):
    codes = _run(2, tmp_path, fail_rank=1)
    assert codes[1] == 3
    assert codes[0] != 0


def test_shard_rows_rejects_uneven_split():
    from ttc_b200.parallel import shard_rows
    with pytest.raises(ValueError):
        shard_rows(torch.zeros(5, 2), 0, 2)
