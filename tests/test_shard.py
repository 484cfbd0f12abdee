"""Multi-rank tests of the time-sharded prefill hand-off.

CPU: gloo ranks (world size 2 and 3) exchange oracle-computed span maps (A_g, B_g) through
``shard.exchange_span_states`` and fold them with ``shard.fold_span_states``; every rank's start
state must equal the sequential oracle's state at its span boundary.
GPU (2 devices, skipped otherwise): NCCL ranks run ``shard.time_sharded_prefill`` end to end and
must match the single-GPU prefill of the whole sequence.
"""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from fixtures import TOL_BF16, baseline_inputs, bf16_round, rel_err


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _span_maps(q, k, v, alpha, beta, lo, hi, initial):
    from oracle import oracle as O
    K = q.shape[3]
    B, _, H, _ = q.shape
    sl = lambda x: x[:, lo:hi]  # noqa: E731
    if initial is not None:  # rank 0: the true scan from the initial state
        _, fin, _ = O.scan_scalar(sl(q), sl(k), sl(v), sl(alpha), sl(beta), initial=initial)
        return None, fin
    eye = np.broadcast_to(np.eye(K), (B, H, K, K)).copy()
    _, A, _ = O.scan_scalar(sl(q), sl(k), np.zeros(sl(k).shape), sl(alpha), sl(beta), initial=eye)
    _, Bs, _ = O.scan_scalar(sl(q), sl(k), sl(v), sl(alpha), sl(beta))
    return A, Bs


def _cpu_worker(rank, world, port, T, result_q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from delta_block_lm_b200 import shard
        B, H, D = 1, 2, 8
        q, k, v, alpha, beta = baseline_inputs(3, B, T, H, D, D)
        init = 0.1 * np.random.default_rng(1).standard_normal((B, H, D, D))
        bounds = [shard.shard_bounds(T, world, g, align=4) for g in range(world)]
        lo, hi = bounds[rank]
        A, Bs = _span_maps(q, k, v, alpha, beta, lo, hi, init if rank == 0 else None)
        if rank == 0:
            As, Bl = shard.exchange_span_states(torch.tensor(Bs), None, rank, world)
        else:
            As, Bl = shard.exchange_span_states(torch.tensor(A), torch.tensor(Bs), rank, world)
        s_in = shard.fold_span_states(Bl[0], As, Bl, rank) if rank > 0 else torch.tensor(init)
        from oracle import oracle as O
        _, ref, _ = O.scan_scalar(q[:, :lo], k[:, :lo], v[:, :lo], alpha[:, :lo], beta[:, :lo],
                                  initial=init) if lo > 0 else (None, init, None)
        result_q.put((rank, float(np.abs(s_in.numpy() - ref).max())))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 3])
def test_time_shard_handoff_gloo(world):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_cpu_worker, args=(r, world, port, 50, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = [q.get(timeout=120) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for rank, err in results:
        assert err < 1e-10, (rank, err)


def test_shard_bounds_cover_and_align():
    from delta_block_lm_b200.shard import shard_bounds
    for n, w, a in ((131072, 8, 64), (1000, 3, 64), (10, 4, 1)):
        b = [shard_bounds(n, w, r, a) for r in range(w)]
        assert b[0][0] == 0 and b[-1][1] == n
        for (l0, h0), (l1, h1) in zip(b, b[1:]):
            assert h0 == l1 and l0 % a == 0


def _gpu_worker(rank, world, port, result_q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev)
    try:
        import delta_block_lm_b200 as dbl
        from delta_block_lm_b200 import shard
        B, T, H, D = 1, 1024, 2, 128
        q, k, v, alpha, beta = baseline_inputs(8, B, T, H, D, D)
        q, k, v = bf16_round(q), bf16_round(k), bf16_round(v)
        tb = lambda x: torch.as_tensor(x).to(dev, torch.bfloat16)  # noqa: E731
        tf = lambda x: torch.as_tensor(x).to(dev, torch.float32)  # noqa: E731
        lo, hi = shard.shard_bounds(T, world, rank, align=64)
        out, fin = shard.time_sharded_prefill(tb(q[:, lo:hi]), tb(k[:, lo:hi]), tb(v[:, lo:hi]),
                                              tf(alpha[:, lo:hi]), tf(beta[:, lo:hi]))
        ref_out, ref_fin = dbl.gdn2_prefill(tb(q), tb(k), tb(v), tf(alpha), tf(beta))
        torch.cuda.synchronize()
        e_out = rel_err(out.float().cpu().numpy(), ref_out[:, lo:hi].float().cpu().numpy())
        e_fin = rel_err(fin.cpu().numpy(), ref_fin.cpu().numpy()) if rank == world - 1 else 0.0
        result_q.put((rank, e_out, e_fin))
    finally:
        dist.destroy_process_group()


@pytest.mark.gpu
def test_time_sharded_prefill_two_gpus(cuda, native_lib):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_gpu_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    results = [q.get(timeout=300) for _ in range(2)]
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    for rank, e_out, e_fin in results:
        # same kernels and inputs; the hand-off adds the f32 fold and one bf16 rounding of S_in
        assert e_out < TOL_BF16 and e_fin < TOL_BF16, (rank, e_out, e_fin)
