"""GPU parity at every BASELINE config's stated shape, against the CPU oracle.

Each test runs the kernel on the whole config (the code path the bench times) and compares a
seeded sample (or all) of its heads / rows with the f64 oracle on the same bf16-rounded inputs.
Every comparison reports three numbers (``fixtures.report``): ``rel_err`` (asserted against the
north star's bound), ``max_rel`` (plain max relative error over elements above 1e-3 rms) and
``ref_pass`` (fraction inside the reference's 2e-5 + 3e-4|e|).  Set DBL_PARITY_REPORT=<file> to
collect them as JSON lines.

  config 0  B2/H4/T512/d64 f32               all heads
  config 1  B8/H16/T4096/d128 bf16            32 of 128 (b, h) heads, seeded
  config 2  256 seq x H16 x 128^2, 64 steps    64 of 4096 (n, h) heads, seeded, every step
  config 3  64 x H16, prefix 4096 + own 1024   all 1024 rows (9 partials merged per row)
  config 4  B1/H16/T131072/d128, segmented     2 of 16 heads over the whole sequence
"""
import numpy as np
import pytest
import torch

import delta_block_lm_b200 as dbl
from fixtures import TOL_BF16, TOL_F32, report
from oracle import oracle as O

pytestmark = pytest.mark.gpu


def host(t):
    return t.detach().float().cpu().numpy()


def _no_device_error(lib):
    import ctypes
    code = ctypes.c_int(0)
    assert lib.dbl_device_error(ctypes.byref(code)) == 0 and code.value == 0, code.value


def test_config0_full(cuda, native_lib):
    g = torch.Generator(device=cuda)
    g.manual_seed(5)
    B, T, H, D = 2, 512, 4, 64
    q = torch.randn((B, T, H, D), device=cuda, generator=g)
    k = torch.randn((B, T, H, D), device=cuda, generator=g)
    q, k = q / q.norm(dim=-1, keepdim=True), k / k.norm(dim=-1, keepdim=True)
    v = torch.randn((B, T, H, D), device=cuda, generator=g)
    beta = torch.sigmoid(torch.randn((B, T, H), device=cuda, generator=g))
    alpha = torch.exp(torch.nn.functional.logsigmoid(3.0 + torch.randn((B, T, H), device=cuda, generator=g)))
    out, fin = dbl.gdn2_prefill(q, k, v, alpha, beta)
    torch.cuda.synchronize()
    ro, rf, _ = O.scan_scalar(host(q), host(k), host(v), host(alpha), host(beta))
    r = report("config0 B2/H4/T512/d64 f32", out=(host(out), ro), final_state=(host(fin), rf))
    assert r["out"]["rel_err"] < TOL_F32 and r["final_state"]["rel_err"] < TOL_F32


def test_config1_full_sampled_heads(cuda, native_lib):
    import bench
    q, k, v, alpha, beta = bench.make_prefill_inputs(torch, cuda, 1234)
    out, fin = dbl.gdn2_prefill(q, k, v, alpha, beta)
    torch.cuda.synchronize()
    _no_device_error(native_lib)
    rng = np.random.default_rng(1)
    pick = rng.choice(8 * 16, size=32, replace=False)
    bs, hs = torch.as_tensor(pick // 16, device=cuda), torch.as_tensor(pick % 16, device=cuda)
    # the sampled heads as a batch of 32 single-head sequences [32, T, 1, D]
    sel = lambda t: host(t[bs, :, hs].unsqueeze(2))  # noqa: E731
    ro, rf, _ = O.scan_scalar(sel(q), sel(k), sel(v), host(alpha[bs, :, hs].unsqueeze(2)),
                              host(beta[bs, :, hs].unsqueeze(2)))
    r = report("config1 B8/H16/T4096/d128 bf16, 32 sampled heads", out=(sel(out), ro),
               final_state=(host(fin[bs, hs].unsqueeze(1)), rf))
    assert r["out"]["rel_err"] < TOL_BF16 and r["final_state"]["rel_err"] < TOL_BF16


def test_config2_full_64_steps(cuda, native_lib):
    n, H, D, steps = 256, 16, 128, 64
    g = torch.Generator(device=cuda)
    g.manual_seed(7)
    state = 0.02 * torch.randn((n, H, D, D), device=cuda, generator=g)
    q = torch.randn((steps, n, H, D), device=cuda, generator=g)
    k = torch.randn((steps, n, H, D), device=cuda, generator=g)
    q = (q / q.norm(dim=-1, keepdim=True)).to(torch.bfloat16)
    k = (k / k.norm(dim=-1, keepdim=True)).to(torch.bfloat16)
    v = torch.randn((steps, n, H, D), device=cuda, generator=g).to(torch.bfloat16)
    beta = torch.sigmoid(torch.randn((steps, n, H), device=cuda, generator=g))
    alpha = torch.exp(torch.nn.functional.logsigmoid(3.0 + torch.randn((steps, n, H), device=cuda, generator=g)))
    rng = np.random.default_rng(2)
    pick = rng.choice(n * H, size=64, replace=False)
    Sref = host(state).reshape(n * H, D, D)[pick].astype(np.float64)
    scale = 1.0 / np.sqrt(D)
    outs, refs = [], []
    for s in range(steps):
        o = dbl.gdn2_decode_step(q[s], k[s], v[s], alpha[s], beta[s], state)
        fl = lambda t, w: host(t).reshape(n * H, w)[pick]  # noqa: E731
        a = np.repeat(host(alpha[s]).reshape(-1, 1)[pick], D, 1)
        b_ = np.repeat(host(beta[s]).reshape(-1, 1)[pick], D, 1)
        ro, Sref = O.step(fl(q[s], D) * scale, fl(k[s], D), fl(v[s], D), a, b_, b_, Sref)
        outs.append(fl(o, D))
        refs.append(ro)
    torch.cuda.synchronize()
    r = report("config2 decode 256x16x128^2, 64 steps, 64 sampled heads",
               out=(np.stack(outs), np.stack(refs)), state=(host(state).reshape(n * H, D, D)[pick], Sref))
    assert r["out"]["rel_err"] < TOL_BF16 and r["state"]["rel_err"] < TOL_BF16


def test_config3_full_all_rows(cuda, native_lib):
    n, H, D, lp, lo = 64, 16, 128, 4096, 1024
    g = torch.Generator(device=cuda)
    g.manual_seed(9)
    mk = lambda *s: torch.randn(s, device=cuda, generator=g).to(torch.bfloat16)  # noqa: E731
    q, kp, vp, ko, vo = mk(n, H, D), mk(H, lp, D), mk(H, lp, D), mk(n, H, lo, D), mk(n, H, lo, D)
    o, m, s = dbl.relay_merge_decode(q, kp, vp, ko, vo)
    torch.cuda.synchronize()
    ro, rm, rs = O.relay_merge(host(q), host(kp), host(vp), host(ko), host(vo), 1.0 / np.sqrt(D))
    r = report("config3 relay 64x16, prefix 4096 + own 1024, all rows", out=(host(o), ro),
               row_max=(host(m), rm), row_sum=(host(s), rs))
    assert r["out"]["rel_err"] < TOL_BF16
    assert r["row_max"]["rel_err"] < TOL_BF16 and r["row_sum"]["rel_err"] < TOL_BF16


def _config4_inputs(dev, t=131072):
    import bench
    return bench.make_prefill_inputs(torch, dev, 777, b=1, t=t)


def _config4_oracle(q, k, v, alpha, beta, heads):
    """The oracle over the whole sequence for the given heads, run as a batch of single-head
    sequences: returns (out [h, T, 1, D], final_state [h, 1, D, D], scores)."""
    hs = list(heads)
    seq = lambda t: host(t[0, :, hs].transpose(0, 1).unsqueeze(2))  # [T,h,D] -> [h,T,1,D]  # noqa: E731
    gate = lambda t: host(t[0, :, hs].transpose(0, 1).unsqueeze(2))  # [T,h] -> [h,T,1]  # noqa: E731
    return O.scan_scalar(seq(q), seq(k), seq(v), gate(alpha), gate(beta))


def test_config4_full_segmented_two_heads(cuda, native_lib):
    from delta_block_lm_b200 import shard
    q, k, v, alpha, beta = _config4_inputs(cuda)
    out, fin = shard.segmented_prefill(q, k, v, alpha, beta)
    torch.cuda.synchronize()
    _no_device_error(native_lib)
    heads = (0, 15)
    ro, rf, _ = _config4_oracle(q, k, v, alpha, beta, heads)
    got_o = np.stack([host(out[0, :, h]) for h in heads])
    got_f = np.stack([host(fin[0, h]) for h in heads])
    r = report("config4 B1/H16/T131072/d128 bf16, 1 GPU segmented, heads 0 and 15",
               out=(got_o, ro[:, :, 0]), final_state=(got_f, rf[:, 0]))
    assert r["out"]["rel_err"] < TOL_BF16 and r["final_state"]["rel_err"] < TOL_BF16


def test_config4_full_time_sharded_devices(cuda, native_lib):
    # the C-ABI multi-device entry (dbl_gdn2_prefill_time_sharded) at full size: two spans on two
    # GPUs when there are two, else both on cuda:0 (the hand-off then copies within one device)
    q, k, v, alpha, beta = _config4_inputs(cuda)
    devs = [torch.device("cuda", 0), torch.device("cuda", 1 if torch.cuda.device_count() > 1 else 0)]
    T = q.shape[1]
    half = T // 2
    spans = []
    for g, dev in enumerate(devs):
        sl = slice(g * half, (g + 1) * half)
        spans.append(tuple(x[:, sl].to(dev).contiguous() for x in (q, k, v, alpha, beta)))
    outs, fin = dbl.gdn2_prefill_time_sharded_devices(spans)
    for d in devs:
        torch.cuda.synchronize(d)
    _no_device_error(native_lib)
    heads = (0, 15)
    ro, rf, _ = _config4_oracle(q, k, v, alpha, beta, heads)
    got_o = np.stack([np.concatenate([host(o[0, :, h]) for o in outs]) for h in heads])
    got_f = np.stack([host(fin[0, h]) for h in heads])
    r = report(f"config4 B1/H16/T131072/d128 bf16, time-sharded over devices {[d.index for d in devs]}, heads 0 and 15",
               out=(got_o, ro[:, :, 0]), final_state=(got_f, rf[:, 0]))
    assert r["out"]["rel_err"] < TOL_BF16 and r["final_state"]["rel_err"] < TOL_BF16


@pytest.mark.parametrize("H", [3, 12])
def test_span_fold_matches_f64(cuda, native_lib, H):
    # H = 3: 16-column blocks.  H = 12, K = V = 128: the composed transition and the offset fold
    # need (8 + 8) x 12 = 192 blocks of 16 columns, more than one wave of 148 SMs, so the launch
    # takes 32-column blocks
    rng = np.random.default_rng(3)
    S, K = 5, 128
    V = 64 if H == 3 else 128
    A = (rng.standard_normal((S, H, K, K)) / np.sqrt(K) * 0.9).astype(np.float32)
    Bm = rng.standard_normal((S, H, K, V)).astype(np.float32)
    x0 = rng.standard_normal((H, K, V)).astype(np.float32)
    t = lambda x: torch.as_tensor(x, device=cuda)  # noqa: E731
    starts, end, comp = dbl.gdn2_span_fold(t(A), t(Bm), t(x0), want_starts=True, want_composed=True)
    torch.cuda.synchronize()
    x = x0.astype(np.float64)
    c = np.broadcast_to(np.eye(K), (H, K, K)).astype(np.float64)
    ref_starts = []
    for s in range(S):
        ref_starts.append(x)
        x = np.einsum("hik,hkv->hiv", A[s].astype(np.float64), x) + Bm[s]
        c = np.einsum("hik,hkj->hij", A[s].astype(np.float64), c)
    r = report(f"span fold S5/H{H}/K128/V{V} f32", starts=(host(starts), np.stack(ref_starts)), end=(host(end), x),
               composed=(host(comp), c))
    for name in ("starts", "end", "composed"):
        assert r[name]["rel_err"] < 1e-5, name


# segments = 8: equal segments.  segments = 0: the lead schedule -- at H = 4 a lead segment of 4
# chunks and 31 segments of 4 (30 map segments, a 30-step fold); at H = 16, T = 4096 a lead
# segment of 10 chunks and 9 segments of 6
@pytest.mark.parametrize("h,t,segments", [(4, 8192, 8), (4, 8192, 0), (16, 4096, 0)])
def test_segmented_prefill_with_masks_and_initial(cuda, native_lib, h, t, segments):
    import bench
    q, k, v, alpha, beta = bench.make_prefill_inputs(torch, cuda, 41, b=1, t=t, h=h)
    g = torch.Generator(device=cuda)
    g.manual_seed(2)
    valid = (torch.rand((1, t), device=cuda, generator=g) > 0.05).float()
    reset = (torch.rand((1, t), device=cuda, generator=g) > 0.998).float()
    init = 0.02 * torch.randn((1, h, 128, 128), device=cuda, generator=g)
    out, fin = dbl.gdn2_prefill_segmented(q, k, v, alpha, beta, segments=segments, valid=valid, reset=reset,
                                          initial_state=init)
    torch.cuda.synchronize()
    _no_device_error(native_lib)
    ro, rf, _ = O.scan_scalar(host(q), host(k), host(v), host(alpha), host(beta), host(valid) > 0,
                              host(reset) > 0, host(init))
    r = report(f"segmented prefill B1/H{h}/T{t} d128 bf16, segments={segments}, masks + initial state",
               out=(host(out), ro), final_state=(host(fin), rf))
    assert r["out"]["rel_err"] < TOL_BF16 and r["final_state"]["rel_err"] < TOL_BF16
    assert np.all(host(out)[0][host(valid)[0] == 0] == 0.0)


def test_time_sharded_graph_one_device(cuda, native_lib):
    # shard.TimeShardedPrefillGraph at world size 1 captures the library's lead schedule (a side
    # stream forked and joined inside the call): replays match the eager call bit for bit, also
    # after new values are copied into the captured inputs
    import bench
    from delta_block_lm_b200 import shard
    q, k, v, alpha, beta = bench.make_prefill_inputs(torch, cuda, 43, b=1, t=16384)
    plan = shard.TimeShardedPrefillGraph(q, k, v, alpha, beta)
    for seed in (43, 44):
        if seed != 43:
            for dst, src in zip((q, k, v, alpha, beta), bench.make_prefill_inputs(torch, cuda, seed, b=1, t=16384)):
                dst.copy_(src)
        go, gf = plan.replay()
        eo, ef = dbl.gdn2_prefill_segmented(q, k, v, alpha, beta)
        torch.cuda.synchronize()
        assert torch.equal(go, eo) and torch.equal(gf, ef)
    plan.release()
    _no_device_error(native_lib)


def test_grouped_segments_one_device(cuda, native_lib):
    # the multi-GPU rank path on one device: a T = 32768 span (a 4-GPU rank's share of config 4)
    # as 8 segments of 57 chunks plus one of 56 (shard.segment_groups; the ninth runs on a side
    # stream), its maps, fold and rescan, eager and captured as a CUDA graph, against the oracle on
    # two heads and against the unsegmented kernel on all heads
    import bench
    from delta_block_lm_b200 import shard
    T = 32768
    q, k, v, alpha, beta = bench.make_prefill_inputs(torch, cuda, 45, b=1, t=T)
    groups = shard.segment_groups(T, 16, shard.sm_count(cuda))
    assert len(groups) == 2 and sum(c for _, c, _ in groups) == 9

    def step():
        maps = shard.segment_maps(q, k, v, alpha, beta, groups=groups)
        return shard.segmented_prefill(q, k, v, alpha, beta, groups=groups, maps=maps)

    out, fin = step()
    torch.cuda.synchronize()
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        step()
    torch.cuda.current_stream().wait_stream(side)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        g_out, g_fin = step()
    graph.replay()
    torch.cuda.synchronize()
    assert torch.equal(g_out, out) and torch.equal(g_fin, fin)
    del graph
    _no_device_error(native_lib)
    p_out, p_fin = dbl.gdn2_prefill(q, k, v, alpha, beta)
    torch.cuda.synchronize()
    r0 = report("grouped segments T32768/H16 (8 x 57 + 56 chunks) vs the unsegmented kernel",
                out=(host(out), host(p_out)), final_state=(host(fin), host(p_fin)))
    assert r0["out"]["rel_err"] < TOL_BF16 and r0["final_state"]["rel_err"] < TOL_BF16
    heads = (0, 15)
    ro, rf, _ = _config4_oracle(q, k, v, alpha, beta, heads)
    got_o = np.stack([host(out[0, :, h]) for h in heads])
    got_f = np.stack([host(fin[0, h]) for h in heads])
    r = report("grouped segments T32768/H16, heads 0 and 15 vs the oracle",
               out=(got_o, ro[:, :, 0]), final_state=(got_f, rf[:, 0]))
    assert r["out"]["rel_err"] < TOL_BF16 and r["final_state"]["rel_err"] < TOL_BF16
