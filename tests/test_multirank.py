"""Head-sharded decode across ranks, and its failure handling, on CPU gloo ranks.

Each rank computes the per-head outputs of its shard with the CPU oracle (the
GPU kernels compute the same per-head values: heads are independent), and the
all-gather must reproduce the unsharded layer.  Failures are made on the host:
a mismatched head partition, a rank that never joins, a rank that exits."""

import os
import socket
import time

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

import starkv_oracle as O
from starkv import dist as sd
from starkv.synthetic import make_layer, make_spec


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _env(rank, world, port):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world))


def _sharded_worker(rank, world, port, q):
    try:
        _env(rank, world, port)
        sd.init("gloo", timeout_s=30)
        spec = make_spec("c1", seed=2, num_q_heads=8, batch=2, context=200)
        data = make_layer(spec)
        sd.check_partition(spec)
        sub = sd.shard_spec(spec, rank, world)
        h0, h1 = sd.head_range(spec, rank, world)
        kv0 = h0 // (spec.num_q_heads // spec.num_kv_heads)
        qz = O.quantize_layer(data.xk, data.xv, spec.context)
        vcol = np.concatenate([[0], np.cumsum(spec.v_ranks)])
        b0 = spec.v_block_of_kv()[kv0]
        b1 = b0 + sub.num_v_blocks
        xk = qz["xk_hat"][kv0:kv0 + sub.num_kv_heads]
        xv = qz["xv_hat"][:, :, vcol[b0]:vcol[b1]]
        v_u = data.v_u[kv0 * 128:(kv0 + sub.num_kv_heads) * 128, vcol[b0]:vcol[b1]]
        out = O.decode_attention(data.q[:, h0:h1], xk, data.k_u[kv0:kv0 + sub.num_kv_heads], xv, v_u,
                                 sub.k_ranks, sub.v_ranks, sub.v_block_of_kv(), O.rope_inv_freq(spec.theta),
                                 128 ** -0.5, dtype=np.float32)
        full = sd.gather_heads(torch.from_numpy(out))
        ref = O.layer_reference(data, dtype=np.float32)
        q.put(("ok", O.rel_l2(full.numpy(), ref)))
        dist.destroy_process_group()
    except Exception as e:  # noqa: BLE001
        q.put(("err", repr(e)))


def _mismatch_worker(rank, world, port, q):
    try:
        _env(rank, world, port)
        sd.init("gloo", timeout_s=30)
        spec = make_spec("c1", seed=2 + rank, num_q_heads=8, batch=1, context=10)   # different ranks per rank
        sd.check_partition(spec)
        q.put(("ok", rank))
    except Exception as e:  # noqa: BLE001
        q.put(("err", repr(e)))
    finally:
        if dist.is_initialized():
            dist.destroy_process_group()


def _leaver_worker(rank, world, port, q):
    try:
        _env(rank, world, port)
        sd.init("gloo", timeout_s=5)
        spec = make_spec("c1", seed=2, num_q_heads=8, batch=1, context=10)
        sd.check_partition(spec)
        if rank == 1:
            q.put(("left", rank))
            time.sleep(0.5)                              # let the queue flush
            os._exit(0)                                  # leaves between steps, nothing in flight
        t0 = time.time()
        sd.gather_heads(torch.zeros(1, 4, 128))
        q.put(("ok", time.time() - t0))
    except Exception as e:  # noqa: BLE001
        q.put(("err", repr(e)))


def _lonely_worker(rank, world, port, q):
    try:
        _env(rank, world, port)
        t0 = time.time()
        sd.init("gloo", timeout_s=5)
        q.put(("ok", time.time() - t0))
    except Exception as e:  # noqa: BLE001
        q.put(("err", repr(e)))


def _run(fn, world=2, timeout=120, nprocs=None):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=fn, args=(r, world, port, q)) for r in range(world if nprocs is None else nprocs)]
    for p in procs:
        p.start()
    res = []
    deadline = time.time() + timeout
    while len(res) < len(procs) and time.time() < deadline:
        try:
            res.append(q.get(timeout=1.0))
        except Exception:  # noqa: BLE001
            if not any(p.is_alive() for p in procs):
                break
    for p in procs:
        p.join(timeout=10)
        if p.is_alive():
            p.kill()
    return res


def test_shard_spec_partitions_heads():
    spec = make_spec("c1")
    for world in (1, 2, 4, 8):
        subs = [sd.shard_spec(spec, r, world) for r in range(world)]
        assert sum(s.num_q_heads for s in subs) == spec.num_q_heads
        assert [r for s in subs for r in s.k_ranks] == spec.k_ranks
        assert [r for s in subs for r in s.v_ranks] == spec.v_ranks
    with pytest.raises(ValueError):
        sd.shard_spec(spec, 0, 3)


def test_uneven_v_blocks_are_rejected():
    """V blocks of different KV-head counts would give ranks different head
    counts; the equal-sized all-gather cannot collect those, so sharding refuses."""
    spec = make_spec("c1", num_q_heads=12, v_block_kv=[4, 8], v_ranks=[64, 128])
    with pytest.raises(ValueError, match="different KV-head counts"):
        sd.shard_spec(spec, 0, 2)
    assert sd.shard_spec(spec, 0, 1).num_q_heads == 12


def test_sharded_decode_gathers_to_the_full_layer():
    res = _run(_sharded_worker)
    oks = [r for r in res if r[0] == "ok"]
    assert oks and not [r for r in res if r[0] == "err"], res
    assert oks[0][1] < 1e-5


def test_mismatched_partition_raises_on_every_rank():
    res = _run(_mismatch_worker)
    assert len(res) == 2 and all(r[0] == "err" and "partition mismatch" in r[1] for r in res), res


def test_rank_that_leaves_makes_the_next_collective_fail():
    res = _run(_leaver_worker, timeout=90)
    survivors = [r for r in res if r[0] != "left"]
    assert survivors and survivors[0][0] == "err", res


def test_rank_that_never_joins_times_out():
    res = _run(_lonely_worker, world=2, nprocs=1, timeout=90)
    assert res and res[0][0] == "err", res
