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


def _gpu_worker(rank, world, port, tmpdir, result_q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev)
    try:
        import bench
        from delta_block_lm_b200 import shard
        # BASELINE config 4 at full size: B1/H16/T131072/d128 bf16, this rank's contiguous span
        q, k, v, alpha, beta = bench.make_prefill_inputs(torch, dev, 777, b=1, t=131072)
        lo, hi = shard.shard_bounds(q.shape[1], world, rank, align=64)
        span = tuple(x[:, lo:hi].contiguous() for x in (q, k, v, alpha, beta))
        out, fin = shard.time_sharded_prefill(*span)
        torch.cuda.synchronize()
        np.save(os.path.join(tmpdir, f"out{rank}.npy"), out[0, :, [0, 15]].float().cpu().numpy())
        if rank == world - 1:
            np.save(os.path.join(tmpdir, "fin.npy"), fin[0, [0, 15]].cpu().numpy())
        # the same step captured as a CUDA graph (all_gather included) replays to the same bits
        plan = shard.TimeShardedPrefillGraph(*span)
        go, gf = plan.replay()
        torch.cuda.synchronize()
        same = bool(torch.equal(go, out) and torch.equal(gf, fin))
        plan.release()
        del plan
        torch.cuda.synchronize()
        result_q.put((rank, lo, hi, same))
    finally:
        dist.destroy_process_group()


@pytest.mark.gpu
def test_time_sharded_prefill_two_gpus(cuda, native_lib, tmp_path):
    # one process per GPU over NCCL (the torchrun layout), config 4 at full size, heads 0 and 15
    # of the whole sequence against the f64 oracle
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    import bench
    from fixtures import report
    from oracle import oracle as O
    ctx = mp.get_context("spawn")
    q_ = ctx.Queue()
    port = _free_port()
    world = 2
    procs = [ctx.Process(target=_gpu_worker, args=(r, world, port, str(tmp_path), q_)) for r in range(world)]
    for p in procs:
        p.start()
    spans = sorted(q_.get(timeout=600) for _ in range(world))
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    assert all(s[3] for s in spans), "graph replay differs from the eager step"
    q, k, v, alpha, beta = bench.make_prefill_inputs(torch, cuda, 777, b=1, t=131072)
    hs = [0, 15]
    seq = lambda t: t[0, :, hs].transpose(0, 1).unsqueeze(2).float().cpu().numpy()  # noqa: E731
    ro, rf, _ = O.scan_scalar(seq(q), seq(k), seq(v), seq(alpha), seq(beta))
    got = np.concatenate([np.load(os.path.join(tmp_path, f"out{s[0]}.npy")) for s in spans], axis=0)
    r = report("config4 B1/H16/T131072/d128 bf16, time-sharded over 2 NCCL ranks, heads 0 and 15",
               out=(got.transpose(1, 0, 2), ro[:, :, 0]), final_state=(np.load(os.path.join(tmp_path, "fin.npy")), rf[:, 0]))
    assert r["out"]["rel_err"] < TOL_BF16 and r["final_state"]["rel_err"] < TOL_BF16


def test_segment_composition_matches_oracle():
    # compose_maps / segment_starts on oracle segment maps reproduce the sequential scan's states.
    from delta_block_lm_b200 import shard
    from oracle import oracle as O
    B, T, H, D, S = 1, 48, 2, 6, 4
    q, k, v, alpha, beta = baseline_inputs(12, B, T, H, D, D)
    L = T // S
    As, Bs = [], []
    for s in range(S):
        sl = slice(s * L, (s + 1) * L)
        eye = np.broadcast_to(np.eye(D), (1, H, D, D)).copy()
        _, A, _ = O.scan_scalar(q[:, sl], k[:, sl], np.zeros(k[:, sl].shape), alpha[:, sl], beta[:, sl], initial=eye)
        _, Bm, _ = O.scan_scalar(q[:, sl], k[:, sl], v[:, sl], alpha[:, sl], beta[:, sl])
        As.append(A[0])
        Bs.append(Bm[0])
    A = torch.tensor(np.stack(As))
    Bm = torch.tensor(np.stack(Bs))
    init = torch.tensor(0.1 * np.random.default_rng(0).standard_normal((1, H, D, D)))
    starts = shard.segment_starts(A, Bm, init)
    At, Bt = shard.compose_maps(A, Bm)
    for s in range(S):
        _, ref, _ = O.scan_scalar(q[:, :s * L], k[:, :s * L], v[:, :s * L], alpha[:, :s * L],
                                  beta[:, :s * L], initial=init.numpy()) if s else (None, init.numpy(), None)
        assert np.abs(starts[s].numpy() - ref[0]).max() < 1e-10
    _, full, _ = O.scan_scalar(q, k, v, alpha, beta, initial=init.numpy())
    assert np.abs((torch.matmul(At, init) + Bt).numpy() - full).max() < 1e-10


def test_segment_groups():
    from delta_block_lm_b200.shard import segment_groups
    # floor(148 / 16) = 9 segments: 8 of ceil(n / 9) chunks and a shorter ninth
    assert segment_groups(32768, 16) == [(0, 8, 57 * 64), (456 * 64, 1, 56 * 64)]
    assert segment_groups(16384, 16) == [(0, 8, 29 * 64), (232 * 64, 1, 24 * 64)]
    assert segment_groups(4096, 16) == [(0, 8, 512)]            # 64 chunks: 8 x 8, no remainder
    assert segment_groups(8192, 4) == [(0, 32, 256)]            # 37 allowed, 32 x 4 chunks cover 128
    assert segment_groups(100, 16) == [(0, 1, 100)]             # not whole chunks
    assert segment_groups(131072, 128) == [(0, 1, 131072)]      # heads already fill the GPU
    for t, h in ((32768, 16), (65536, 16), (16384, 16), (8192, 4), (640, 16), (64 * 7, 3)):
        g = segment_groups(t, h)
        assert sum(c * l for _, c, l in g) == t and sum(c for _, c, _ in g) * h <= 148
        assert all(l % 64 == 0 for _, _, l in g)
        assert all(t0 == g[0][1] * g[0][2] for t0, _, _ in g[1:])


def test_pick_segments():
    from delta_block_lm_b200.shard import pick_segments
    assert pick_segments(131072, 16) == 8      # 128 CTAs on 148 SMs
    assert pick_segments(16384, 16) == 8
    assert pick_segments(4096, 16) == 8
    assert pick_segments(100, 16) == 1          # not whole chunks
    assert pick_segments(131072, 128) == 1      # heads already fill the GPU


@pytest.mark.gpu
def test_segmented_prefill_matches_single_scan(cuda, native_lib):
    import delta_block_lm_b200 as dbl
    from delta_block_lm_b200 import shard
    B, T, H, D = 1, 4096, 2, 128
    q, k, v, alpha, beta = baseline_inputs(31, B, T, H, D, D)
    q, k, v = bf16_round(q), bf16_round(k), bf16_round(v)
    tb = lambda x: torch.as_tensor(x).to(cuda, torch.bfloat16)  # noqa: E731
    tf = lambda x: torch.as_tensor(x).to(cuda, torch.float32)  # noqa: E731
    init = tf(0.02 * np.random.default_rng(3).standard_normal((1, H, D, D)))
    out, fin = shard.segmented_prefill(tb(q), tb(k), tb(v), tf(alpha), tf(beta), initial_state=init)
    ref_out, ref_fin = dbl.gdn2_prefill(tb(q), tb(k), tb(v), tf(alpha), tf(beta), initial_state=init)
    torch.cuda.synchronize()
    assert shard.pick_segments(T, H) > 1
    assert rel_err(out.float().cpu().numpy(), ref_out.float().cpu().numpy()) < TOL_BF16
    assert rel_err(fin.cpu().numpy(), ref_fin.cpu().numpy()) < TOL_BF16
