"""The N>1 path on CPU: world_size-2 gloo ranks each compute their shard of
(batch, head) slices (the oracle stands in for the per-GPU kernel) and the
validation gather reassembles the result on rank 0; a rank that leaves early
makes the others fail with an error within the process-group timeout instead
of hanging."""
import datetime
import os
import socket
import sys

import numpy as np
import pytest

torch = pytest.importorskip("torch")
import torch.distributed as dist  # noqa: E402
import torch.multiprocessing as mp  # noqa: E402

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _init(rank, world, port, timeout_s=60):
    sys.path.insert(0, ROOT)
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=timeout_s))
    import __graft_entry__ as ge
    ge.package()
    from mlir_flashattention_b200 import sharding, workloads
    return ge, sharding, workloads


def _shard_worker(rank, world, port, out_path):
    ge, sharding, wl = _init(rank, world, port)
    o = ge.oracle()
    w = wl.Workload("t", "f32", 2, 4, 2, 256, 32, True, seed=3)
    inp = wl.make_inputs(w)
    a, b = sharding.shard_groups(w.B, w.Hkv, world, rank)
    group = w.Hq // w.Hkv
    flat = inp.qf.reshape(w.B * w.Hkv, group, w.N, w.D)
    kf = inp.kf.reshape(w.B * w.Hkv, 1, w.N, w.D)
    vf = inp.vf.reshape(w.B * w.Hkv, 1, w.N, w.D)
    O, L = o.attn_batched(flat[a:b], kf[a:b], vf[a:b], w.scale, causal=True, nthreads=1)
    parts = sharding.gather_rows(torch.from_numpy(O), world, rank)
    if rank == 0:
        full = torch.cat(parts).numpy().reshape(w.B, w.Hq, w.N, w.D)
        ref, _ = o.attn_batched(inp.qf, inp.kf, inp.vf, w.scale, causal=True, nthreads=1)
        np.save(out_path, np.array([float(np.abs(full - ref).max())]))
    dist.barrier()
    dist.destroy_process_group()


def _rank_values_worker(rank, world, port, out_path):
    _, sharding, _ = _init(rank, world, port)
    vals = sharding.rank_values(1.5 + rank, world)
    if rank == 0:
        np.save(out_path, np.array(vals))
    dist.barrier()
    dist.destroy_process_group()


def _early_exit_worker(rank, world, port, out_path):
    _, sharding, _ = _init(rank, world, port, timeout_s=5)
    if rank == 1:
        os._exit(0)  # leaves between steps, before the gather
    try:
        sharding.gather_rows(torch.zeros(4, 2), world, rank)
        result = "completed"
    except Exception as e:  # noqa: BLE001
        result = "error:" + type(e).__name__
    with open(out_path, "w") as f:
        f.write(result)
    os._exit(0)


def test_shards_gather_to_full_result(tmp_path):
    out = str(tmp_path / "err.npy")
    mp.spawn(_shard_worker, args=(2, _port(), out), nprocs=2, join=True)
    assert np.load(out)[0] == 0.0


def test_rank_times_gathered_in_rank_order(tmp_path):
    """The bench's max-over-ranks time: every rank's duration reaches every
    rank, in rank order."""
    out = str(tmp_path / "vals.npy")
    mp.spawn(_rank_values_worker, args=(2, _port(), out), nprocs=2, join=True)
    assert np.load(out).tolist() == [1.5, 2.5]


def test_rank_leaving_early_is_detected(tmp_path):
    out = str(tmp_path / "res.txt")
    ctx = mp.spawn(_early_exit_worker, args=(2, _port(), out), nprocs=2, join=False)
    ok = False
    for _ in range(4):  # rank 0 must give up within its 5 s process-group timeout
        ok = ctx.join(timeout=30)
        if ok:
            break
    if not ok:
        for p in ctx.processes:
            p.kill()
    assert ok, "surviving rank did not detect the departed rank"
    assert open(out).read().startswith("error:")
