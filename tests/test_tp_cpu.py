"""Tensor-parallel sharding on the CPU (no GPU): world-size-2, -4 and -8 gloo ranks each
take their shard of the Q4_0 weights with torchnative_b200.tp, run the oracle
(the reference's CPU arithmetic) on it, and all-gather; the gathered rows equal
the unsharded oracle output bit for bit, because a column shard changes which
rank computes an output, never how."""

import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from oracle import oracle
from tests import q4_exact
from torchnative_b200 import tp as tpm


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _blob(rng, n, k) -> torch.Tensor:
    return torch.frombuffer(bytearray(q4_exact.random_q4_0_blob(rng, n, k)), dtype=torch.uint8)


def _gather_np(group, arr: np.ndarray, world: int) -> np.ndarray:
    """rank-major concatenation along the last axis, through TPGroup.all_gather."""
    rows, c = arr.shape
    local = torch.from_numpy(np.ascontiguousarray(arr))
    full = torch.empty(world * rows * c, dtype=local.dtype)
    group.all_gather(full, local)
    return full.view(world, rows, c).permute(1, 0, 2).reshape(rows, world * c).numpy()


def _worker(rank, world, port, failures):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        g = tpm.TPGroup(rank, world, None)
        rng = np.random.default_rng(5)  # same weights and inputs on every rank
        # at least one KV head per rank
        B, H, I, D = 2, 256, 512, 32
        Hkv = max(4, world)
        Hq = 2 * Hkv
        x = rng.standard_normal((B, H)).astype(np.float32)
        # column-sharded linear (o / down / lm_head)
        w = _blob(rng, H, H)
        local = tpm.shard_rows(w, H, H, rank, world)
        y_l = oracle.q4_0_linear(x, local.numpy().tobytes(), H // world)
        y = _gather_np(g, y_l, world)
        assert np.array_equal(y, oracle.q4_0_linear(x, w.numpy().tobytes(), H)), "row shards"
        # interleaved gate/up pairs
        gu = _blob(rng, 2 * I, H)
        gu_l = tpm.shard_gate_up_pairs(gu, I, H, rank, world)
        full = oracle.q4_0_linear(x, gu.numpy().tobytes(), 2 * I)
        part = oracle.q4_0_linear(x, gu_l.numpy().tobytes(), 2 * I // world)
        c = 2 * I // world
        assert np.array_equal(part, full[:, rank * c:(rank + 1) * c]), "gate/up pairs"
        # fused q/k/v of this rank's KV-head group, then attention on the local heads
        n = (Hq + 2 * Hkv) * D
        qkv = _blob(rng, n, H)
        qkv_l = tpm.shard_qkv(qkv, Hq, Hkv, D, H, rank, world)
        full = oracle.q4_0_linear(x, qkv.numpy().tobytes(), n)
        part = oracle.q4_0_linear(x, qkv_l.numpy().tobytes(), n // world)
        hq, hkv = Hq // world, Hkv // world
        q_f, k_f, v_f = full[:, :Hq * D], full[:, Hq * D:(Hq + Hkv) * D], full[:, (Hq + Hkv) * D:]
        assert np.array_equal(part[:, :hq * D], q_f[:, rank * hq * D:(rank + 1) * hq * D])
        assert np.array_equal(part[:, hq * D:(hq + hkv) * D], k_f[:, rank * hkv * D:(rank + 1) * hkv * D])
        assert np.array_equal(part[:, (hq + hkv) * D:], v_f[:, rank * hkv * D:(rank + 1) * hkv * D])
        S = 40
        kc = rng.standard_normal((B, Hkv, S, D)).astype(np.float32)
        vc = rng.standard_normal((B, Hkv, S, D)).astype(np.float32)
        q = q_f.reshape(B, Hq, 1, D)
        o_full, _ = oracle.sdpa(q, kc, vc, dtype="float32")
        o_l, _ = oracle.sdpa(np.ascontiguousarray(q[:, rank * hq:(rank + 1) * hq]),
                             np.ascontiguousarray(kc[:, rank * hkv:(rank + 1) * hkv]),
                             np.ascontiguousarray(vc[:, rank * hkv:(rank + 1) * hkv]), dtype="float32")
        o = _gather_np(g, o_l.reshape(B, hq * D), world)
        assert np.array_equal(o, o_full.reshape(B, Hq * D)), "KV-head-group attention"
        # row-parallel o_proj / down_proj (the rowwise plan): rank r's input
        # features [r K/G, (r+1) K/G) -- its own heads' attention output -- give
        # an f32 partial; the partials summed in rank order stay within the
        # counted bound of the unsharded linear, with G more additions
        K = Hq * D
        wo = _blob(rng, H, K)
        wo_l = tpm.shard_cols(wo, H, K, rank, world)
        xo = o_full.reshape(B, K)
        kc_ = K // world
        part = oracle.q4_0_linear(np.ascontiguousarray(xo[:, rank * kc_:(rank + 1) * kc_]), wo_l.numpy().tobytes(), H)
        parts = _gather_np(g, part, world).reshape(B, world, H)
        y = np.zeros((B, H), dtype=np.float32)
        for r_ in range(world):
            y = (y + parts[:, r_]).astype(np.float32)
        exact, abs_sum, ref_err = q4_exact.exact_linear_q4_0(oracle.q8_0_quantize(xo), wo.numpy().tobytes(), B, H, K)
        bound = q4_exact.linear_bound(K + 32 * world, abs_sum, ref_err)
        assert float(np.max(np.abs(y.astype(np.float64) - exact) / bound)) <= 1.0, "row-parallel partial sums"
        # every output row's blocks are split, none re-encoded
        assert np.array_equal(wo_l.numpy().reshape(H, K // 32 // world, 18),
                              wo.numpy().reshape(H, K // 32, 18)[:, rank * (K // 32 // world):(rank + 1) * (K // 32 // world)])
    except AssertionError as e:
        failures.put(f"rank {rank}: {e}")
        raise
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 4, 8])
def test_gloo_ranks_rebuild_the_unsharded_outputs(world):
    ctx = mp.get_context("spawn")
    failures = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, failures)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=180)
    msgs = []
    while not failures.empty():
        msgs.append(failures.get())
    assert not msgs, msgs
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]


def test_shard_refusals():
    w = torch.zeros(10 * 18, dtype=torch.uint8)
    with pytest.raises(ValueError, match="does not divide"):
        tpm.shard_rows(w, 10, 32, 0, 4)
    with pytest.raises(ValueError, match="whole 32-element blocks"):
        tpm.row_slice(w, 10, 40, 0, 1)
    with pytest.raises(ValueError, match="is not"):
        tpm.row_slice(w[:-1], 10, 32, 0, 1)
    assert tpm.shard_rows(w, 10, 32, 1, 2).numel() == 5 * 18
    w2 = torch.zeros(2 * 3 * 18, dtype=torch.uint8)
    with pytest.raises(ValueError, match="does not divide"):
        tpm.shard_cols(w2, 2, 96, 0, 2)  # 3 blocks per row over 2 ranks
    assert tpm.shard_cols(w2, 2, 96, 2, 3).numel() == 2 * 18


def _leaving_worker(rank, world, port, result):
    """Rank 1 joins the group, passes one barrier and leaves before the
    gather; rank 0's gather must end with PeerLost, not hang."""
    import datetime

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=5))
    dist.barrier()
    if rank == 1:
        os._exit(0)  # gone between steps, with nothing in flight
    g = tpm.TPGroup(rank, world, None)
    try:
        g.all_gather(torch.empty(2 * 8), torch.ones(8))
        result.put("no error")
    except tpm.PeerLost as e:
        result.put("PeerLost: " + str(e))
    except Exception as e:  # noqa: BLE001 -- reported to the parent
        result.put(f"{type(e).__name__}: {e}")
    os._exit(0)


def test_a_rank_that_leaves_before_a_gather_is_named_on_the_host():
    ctx = mp.get_context("spawn")
    result = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_leaving_worker, args=(r, 2, port, result)) for r in range(2)]
    for p in procs:
        p.start()
    try:
        msg = result.get(timeout=60)
    finally:
        for p in procs:
            p.join(timeout=30)
            if p.is_alive():
                p.kill()
    assert msg.startswith("PeerLost"), msg
    assert "rank 0 of 2" in msg
