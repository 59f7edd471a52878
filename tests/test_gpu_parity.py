"""The CUDA path through the C ABI against the oracle (bit-exact where the
north star asks for it: synthetic data, dequantised weights, router logits,
expert ids, dispatch; within a stated tolerance for the FFN and combine)."""
import numpy as np
import pytest

import obsmoe
import oracle as O

pytestmark = pytest.mark.gpu

# FFN / combine outputs: max |gpu - oracle| <= REL * max |oracle| (north star: 1e-2 in bf16)
REL = 1e-2
# against the oracle run in the GEMM path's own arithmetic (bf16 weights): within about one bf16
# ulp of the largest output (2^-8 relative), i.e. only accumulation order differs
REL_SAME = 5e-3


def rel_err(got, ref):
    got = got.astype(np.float32)
    ref = ref.astype(np.float32)
    return float(np.abs(got - ref).max() / max(np.abs(ref).max(), 1e-30))


# ------------------------------------------------------------------ plumbing
def dev(torch, a):
    a = np.ascontiguousarray(a)
    if a.dtype == np.uint16:
        return torch.from_numpy(a.view(np.int16)).cuda()
    if a.dtype == np.uint32:
        return torch.from_numpy(a.view(np.int32)).cuda()
    return torch.from_numpy(a).cuda()


def host(t, dtype):
    t = t.detach().cpu().contiguous()
    return t.numpy().view(dtype)


def empty(torch, shape, dtype):
    tdt = {np.uint16: torch.int16, np.float32: torch.float32, np.int32: torch.int32}[dtype]
    return torch.empty(shape, dtype=tdt, device="cuda")


class Env:
    """A context holding one oracle-generated layer, loaded from host memory."""

    def __init__(self, torch, E, I, K, max_tokens, seed):
        self.torch = torch
        self.shape = obsmoe.MoeShape(2048, I, E, K, n_layers=1, max_tokens=max_tokens)
        self.ctx = obsmoe.MoeContext(self.shape, 0)
        self.L = O.synth_layer(seed, 0, E=E, H=2048, I=I, K=K)
        self.ctx.load_layer(0, self.L)
        self.seed = seed

    def x(self, T, row0=0, seed=None):
        return O.synth_x(self.seed if seed is None else seed, 0, T, 2048, row0=row0)


@pytest.fixture(scope="module")
def small(cuda):
    env = Env(cuda, E=16, I=256, K=4, max_tokens=256, seed=5)
    yield env
    env.ctx.check_device()
    env.ctx.close()


@pytest.fixture(scope="module")
def full(cuda):
    env = Env(cuda, E=128, I=768, K=8, max_tokens=512, seed=0)
    yield env
    env.ctx.check_device()
    env.ctx.close()


# ------------------------------------------------------------- synthetic data
def test_device_activations_match_oracle(cuda):
    for T, row0 in [(1, 0), (37, 5), (512, 0)]:
        x = empty(cuda, (T, 2048), np.uint16)
        obsmoe.synth_activations(3, 1, row0, T, 2048, x)
        cuda.cuda.synchronize()
        assert np.array_equal(host(x, np.uint16), O.synth_x(3, 1, T, 2048, row0=row0))


def test_device_weights_match_oracle(cuda):
    # layer 1 generated on the device from (seed, layer 1); layer 0 loaded from the
    # oracle's host generator for (seed, layer 1): identical router logits and GEMM outputs
    shape = obsmoe.MoeShape(2048, 256, 16, 4, n_layers=2, max_tokens=64)
    ctx = obsmoe.MoeContext(shape, 0)
    L = O.synth_layer(8, 1, E=16, H=2048, I=256, K=4)
    ctx.load_layer(0, L)
    ctx.synth_layer(1, 8)
    x = dev(cuda, O.synth_x(8, 1, 64, 2048))
    a, b = empty(cuda, (64, 16), np.float32), empty(cuda, (64, 16), np.float32)
    ctx.gate_gpu(0, x, a, 64)
    ctx.gate_gpu(1, x, b, 64)
    ya, yb = empty(cuda, (64, 256), np.float32), empty(cuda, (64, 256), np.float32)
    for proj in range(3):
        n_in = 256 if proj == 2 else 2048
        n_out = 2048 if proj == 2 else 256
        xin = dev(cuda, O.synth_x(8, 1, 64, n_in) if n_in == 2048 else O.synth_x(8, 1, 64, 2048)[:, :256])
        ya, yb = empty(cuda, (64, n_out), np.float32), empty(cuda, (64, n_out), np.float32)
        for e in (0, 15):
            ctx.matmul_raw_f32(0, proj, e, xin, 64, ya)
            ctx.matmul_raw_f32(1, proj, e, xin, 64, yb)
            cuda.cuda.synchronize()
            assert cuda.equal(ya, yb)
    cuda.cuda.synchronize()
    assert cuda.equal(a, b)
    ctx.check_device()
    ctx.close()


# -------------------------------------------------------------------- router
@pytest.mark.parametrize("T", [1, 5, 16, 17, 64, 200])
def test_router_logits_bit_exact(small, T):
    torch = small.torch
    x = small.x(T)
    logits = empty(torch, (T, 16), np.float32)
    small.ctx.gate_gpu(0, dev(torch, x), logits, T)
    got = host(logits, np.float32)
    ref = O.router_logits(small.L, x)
    assert np.array_equal(got.view(np.uint32), ref.view(np.uint32))


@pytest.mark.parametrize("T", [1, 512])
def test_router_logits_bit_exact_full(full, T):
    torch = full.torch
    x = full.x(T)
    logits = empty(torch, (T, 128), np.float32)
    full.ctx.gate_gpu(0, dev(torch, x), logits, T)
    ref = O.router_logits(full.L, x)
    assert np.array_equal(host(logits, np.float32).view(np.uint32), ref.view(np.uint32))


def test_route_ids_exact_with_ties_and_bias(small):
    torch = small.torch
    rng = np.random.default_rng(0)
    T = 64
    logits = rng.standard_normal((T, 16)).astype(np.float32)
    logits[3] = 0.0                      # all tied
    logits[4, [1, 7, 9, 12]] = 5.0       # a four-way tie at the top
    bias = (rng.standard_normal(16) * 0.5).astype(np.float32)
    for b in (None, bias):
        ids = empty(torch, (T, 4), np.int32)
        w = empty(torch, (T, 4), np.float32)
        small.ctx.route(dev(torch, logits), T, ids, w, bias=None if b is None else dev(torch, b))
        rid, rw = O.topk(logits, 4, bias=b)
        assert np.array_equal(host(ids, np.int32), rid)
        assert np.allclose(host(w, np.float32), rw, rtol=1e-5, atol=1e-7)
    ids = empty(torch, (T, 4), np.int32)
    w = empty(torch, (T, 4), np.float32)
    small.ctx.route(dev(torch, logits), T, ids, w)
    assert list(host(ids, np.int32)[3]) == [0, 1, 2, 3]
    assert list(host(ids, np.int32)[4]) == [1, 7, 9, 12]


# ------------------------------------------------------------------ dispatch
@pytest.mark.parametrize("case", ["random", "hot", "T1"])
def test_dispatch_exact(small, case):
    torch = small.torch
    rng = np.random.default_rng(1)
    T = {"random": 200, "hot": 100, "T1": 1}[case]
    if case == "hot":   # experts 0..3 get every token, 4..15 none (empty segments)
        ids = np.tile(np.arange(4, dtype=np.int32), (T, 1))
    else:
        ids = np.stack([rng.permutation(16)[:4] for _ in range(T)]).astype(np.int32)
    counts, seg, slot_of = empty(torch, 16, np.int32), empty(torch, 17, np.int32), empty(torch, (T, 4), np.int32)
    small.ctx.dispatch(dev(torch, ids), T, counts, seg, slot_of)
    rc, roff, rslot, _ = O.dispatch(ids, 16)
    c, s, so = host(counts, np.int32), host(seg, np.int32), host(slot_of, np.int32)
    assert np.array_equal(c, rc)
    pad = (rc + 15) // 16 * 16
    assert np.array_equal(s[:16], np.concatenate([[0], np.cumsum(pad)[:-1]]))
    assert s[16] == pad.sum()
    # rank of each (token, k) inside its expert segment equals the oracle's
    assert np.array_equal(so - s[ids], rslot - roff[ids])


def test_dispatch_rejects_bad_ids(small):
    torch = small.torch
    ids = np.array([[0, 1, 2, 99]], np.int32)
    small.ctx.dispatch(dev(torch, ids), 1)
    with pytest.raises(obsmoe.ObsError):
        small.ctx.check_device()
    small.ctx.check_device()  # flag cleared


# --------------------------------------------------------------------- GEMM
@pytest.mark.parametrize("proj", [0, 1, 2])
def test_gemm_dequant_bit_exact(small, proj):
    """One-hot rows through the tcgen05 GEMM read back the in-smem dequant:
    bf16(fma(q, s, b)) for every weight, bit for bit."""
    torch = small.torch
    L = small.L
    in_f = 256 if proj == 2 else 2048
    w, s, b = [(L.gate_w, L.gate_s, L.gate_b), (L.up_w, L.up_s, L.up_b), (L.down_w, L.down_s, L.down_b)][proj]
    e = 11
    ref = O.bf16_to_f32(O.dequant4_bf16(w[e], s[e], b[e]))   # [out, in]
    c0 = 128 if proj != 2 else 0
    n = min(256, in_f)
    eye = np.zeros((n, in_f), np.float32)
    eye[np.arange(n), c0 + np.arange(n)] = 1.0
    y = empty(torch, (n, ref.shape[0]), np.float32)
    small.ctx.matmul_raw_f32(0, proj, e, dev(torch, O.f32_to_bf16(eye)), n, y)
    got = host(y, np.float32)
    assert np.array_equal(got.view(np.uint32), ref[:, c0:c0 + n].T.copy().view(np.uint32))


# bf16 bit patterns of scales at and around the edges of the GEMM's one-instruction unpack
# (exponent field 1..121): zero, subnormal, smallest normal, just under and at 2^-5,
# large, and negative ones on both sides
EDGE_SCALES = np.array([0x0000, 0x0001, 0x007F, 0x0080, 0x3CFF, 0x3D00, 0x3DCC, 0x3F80, 0x4040,
                        0x8080, 0xBC23, 0xBD00, 0xBF00, 0x3C23, 0x3B80, 0x3A00], np.uint16)


@pytest.fixture(scope="module")
def edge(cuda):
    """The small layer with every weight group's scale drawn from EDGE_SCALES (mixed within
    each 32-row warp), so both unpack forms and the per-row choice between them run."""
    env = Env.__new__(Env)
    env.torch = cuda
    env.shape = obsmoe.MoeShape(2048, 256, 16, 4, n_layers=1, max_tokens=256)
    env.ctx = obsmoe.MoeContext(env.shape, 0)
    L = O.synth_layer(5, 0, E=16, H=2048, I=256, K=4)
    rng = np.random.default_rng(17)
    for name in ("gate_s", "up_s", "down_s"):
        a = getattr(L, name)
        setattr(L, name, EDGE_SCALES[rng.integers(0, len(EDGE_SCALES), a.shape)].astype(a.dtype))
    env.L = L
    env.seed = 5
    env.ctx.load_layer(0, L)
    yield env
    env.ctx.check_device()
    env.ctx.close()


@pytest.mark.parametrize("proj", [0, 1, 2])
def test_gemm_dequant_bit_exact_edge_scales(edge, proj):
    """As above, on scales outside the one-instruction unpack's range (and zero / subnormal)."""
    torch = edge.torch
    L = edge.L
    in_f = 256 if proj == 2 else 2048
    w, s, b = [(L.gate_w, L.gate_s, L.gate_b), (L.up_w, L.up_s, L.up_b), (L.down_w, L.down_s, L.down_b)][proj]
    for e in (2, 11):
        ref = O.bf16_to_f32(O.dequant4_bf16(w[e], s[e], b[e]))
        for c0 in range(0, in_f, 256):
            eye = np.zeros((256, in_f), np.float32)
            eye[np.arange(256), c0 + np.arange(256)] = 1.0
            y = empty(torch, (256, ref.shape[0]), np.float32)
            edge.ctx.matmul_raw_f32(0, proj, e, dev(torch, O.f32_to_bf16(eye)), 256, y)
            got = host(y, np.float32)
            assert np.array_equal(got.view(np.uint32), ref[:, c0:c0 + 256].T.copy().view(np.uint32)), (e, c0)


@pytest.mark.parametrize("path,T", [(obsmoe.PATH_DECODE, 3), (obsmoe.PATH_PREFILL, 100)])
def test_expert_ffn_edge_scales_vs_oracle(edge, path, T):
    """Both FFN paths with edge-case scales against the oracle."""
    torch = edge.torch
    x = edge.x(T, row0=3)
    rng = np.random.default_rng(T + 1)
    ids = np.stack([rng.permutation(16)[:4] for _ in range(T)]).astype(np.int32)
    y = empty(torch, (T * 4, 2048), np.uint16)
    edge.ctx.expert_ffn(0, dev(torch, x), dev(torch, ids), T, y, path=path)
    wmode = 0 if path == obsmoe.PATH_DECODE else 1
    _, _, ry = O.moe_ffn_combine(edge.L, x, ids, np.full((T, 4), 0.25, np.float32), wmode=wmode, want_y=True)
    got = O.bf16_to_f32(host(y, np.uint16)).reshape(T, 4, 2048)
    assert rel_err(got, O.bf16_to_f32(ry)) < REL_SAME


@pytest.mark.parametrize("n", [1, 16, 100, 256])
def test_gemm_random_vs_oracle(small, n):
    torch = small.torch
    L = small.L
    x = small.x(n, row0=50)
    W = O.bf16_to_f32(O.dequant4_bf16(L.up_w[3], L.up_s[3], L.up_b[3]))
    ref = O.bf16_to_f32(x).astype(np.float64) @ W.T.astype(np.float64)
    y = empty(torch, (n, 256), np.float32)
    small.ctx.matmul_raw_f32(0, 1, 3, dev(torch, x), n, y)
    assert rel_err(host(y, np.float32), ref) < 1e-5


# ---------------------------------------------------------------- expert FFN
@pytest.mark.parametrize("path,T", [(obsmoe.PATH_DECODE, 1), (obsmoe.PATH_DECODE, 9), (obsmoe.PATH_PREFILL, 1),
                                    (obsmoe.PATH_PREFILL, 77), (obsmoe.PATH_PREFILL, 256)])
def test_expert_ffn_vs_oracle(small, path, T):
    torch = small.torch
    x = small.x(T, row0=7)
    rng = np.random.default_rng(T)
    ids = np.stack([rng.permutation(16)[:4] for _ in range(T)]).astype(np.int32)
    y = empty(torch, (T * 4, 2048), np.uint16)
    small.ctx.expert_ffn(0, dev(torch, x), dev(torch, ids), T, y, path=path)
    wmode = 0 if path == obsmoe.PATH_DECODE else 1
    _, _, ry = O.moe_ffn_combine(small.L, x, ids, np.full((T, 4), 0.25, np.float32), wmode=wmode, want_y=True)
    got = O.bf16_to_f32(host(y, np.uint16)).reshape(T, 4, 2048)
    assert rel_err(got, O.bf16_to_f32(ry)) < REL_SAME


# ---------------------------------------------------------------- the layer
def run_forward(env, x, path, residual=None, bias=None):
    torch = env.torch
    T = x.shape[0]
    out = empty(torch, (T, 2048), np.uint16)
    env.ctx.moe_forward(0, dev(torch, x), out, T, residual=None if residual is None else dev(torch, residual),
                        bias=None if bias is None else dev(torch, bias), path=path)
    return host(out, np.uint16)


def test_config0_decode_vs_oracle(full):
    """Config 0: one Qwen3-30B-A3B MoE layer, decode of one token, seed 0."""
    x = full.x(1)
    got = run_forward(full, x, obsmoe.PATH_AUTO)
    ref, rid, _ = O.moe_layer(full.L, x, wmode=0)
    assert rel_err(O.bf16_to_f32(got), O.bf16_to_f32(ref)) < REL


def test_config1_prefill_vs_oracle(full):
    """Config 1: the same layer, batched prefill of T=512 tokens."""
    x = full.x(512)
    got = run_forward(full, x, obsmoe.PATH_AUTO)
    ref, _, _ = O.moe_layer(full.L, x, wmode=0)
    assert rel_err(O.bf16_to_f32(got), O.bf16_to_f32(ref)) < REL
    ref1, _, _ = O.moe_layer(full.L, x, wmode=1)   # the GEMM path's own arithmetic: much tighter
    assert rel_err(O.bf16_to_f32(got), O.bf16_to_f32(ref1)) < REL_SAME


@pytest.mark.parametrize("T", [2, 17, 64])
def test_decode_and_prefill_paths_agree(small, T):
    x = small.x(T, row0=3)
    a = run_forward(small, x, obsmoe.PATH_DECODE)
    b = run_forward(small, x, obsmoe.PATH_PREFILL)
    assert rel_err(O.bf16_to_f32(a), O.bf16_to_f32(b)) < REL


@pytest.mark.parametrize("path", [obsmoe.PATH_DECODE, obsmoe.PATH_PREFILL])
def test_residual_and_skewed_bias(small, path):
    T = 33 if path == obsmoe.PATH_PREFILL else 4
    x = small.x(T, row0=11)
    res = small.x(T, row0=100)
    bias = np.zeros(16, np.float32)
    bias[6] = 50.0     # expert 6 receives every token
    got = run_forward(small, x, path, residual=res, bias=bias)
    ref, rid, _ = O.moe_layer(small.L, x, bias=bias, residual=res, wmode=0)
    assert np.all(rid[:, 0] == 6)
    assert rel_err(O.bf16_to_f32(got), O.bf16_to_f32(ref)) < REL


def test_max_tokens_and_empty(small):
    x = small.x(256)
    got = run_forward(small, x, obsmoe.PATH_PREFILL)
    ref, _, _ = O.moe_layer(small.L, x, wmode=1)
    assert rel_err(O.bf16_to_f32(got), O.bf16_to_f32(ref)) < REL_SAME
    out = small.torch.empty((1, 2048), dtype=small.torch.int16, device="cuda")
    small.ctx.moe_forward(0, out, out, 0)   # T = 0 is a no-op


def test_host_entry_matches_device(small):
    torch = small.torch
    x = small.x(40, row0=9)
    dev_out = run_forward(small, x, obsmoe.PATH_PREFILL)
    xh = torch.from_numpy(x.view(np.int16)).pin_memory()
    oh = torch.empty((40, 2048), dtype=torch.int16).pin_memory()
    small.ctx.moe_forward_host(0, xh, oh, 40, path=obsmoe.PATH_PREFILL)
    assert np.array_equal(oh.numpy().view(np.uint16), dev_out)


def test_host_async_matches_sync(small):
    """Five pipelined asynchronous host calls (alternating staging slots, some with a residual,
    both paths) give the synchronous host entry's results bit for bit."""
    torch = small.torch
    cases = [(40, obsmoe.PATH_PREFILL, False), (17, obsmoe.PATH_PREFILL, True), (3, obsmoe.PATH_DECODE, False),
             (100, obsmoe.PATH_PREFILL, True), (1, obsmoe.PATH_AUTO, True)]
    ins, want = [], []
    for i, (T, path, with_res) in enumerate(cases):
        xh = torch.from_numpy(small.x(T, row0=11 * i).view(np.int16)).pin_memory()
        rh = torch.from_numpy(small.x(T, row0=5 + 7 * i, seed=9).view(np.int16)).pin_memory() if with_res else None
        oh = torch.empty((T, 2048), dtype=torch.int16).pin_memory()
        small.ctx.moe_forward_host(0, xh, oh, T, residual_host=rh, path=path)
        ins.append((T, path, xh, rh))
        want.append(oh.numpy().copy())
    stream = torch.cuda.Stream()
    outs = [torch.full((T, 2048), -1, dtype=torch.int16).pin_memory() for (T, _, _, _) in ins]
    for (T, path, xh, rh), oh in zip(ins, outs):
        small.ctx.moe_forward_host_async(0, xh, oh, T, residual_host=rh, path=path, stream=stream)
    small.ctx.host_join(stream)
    stream.synchronize()
    for oh, w in zip(outs, want):
        assert np.array_equal(oh.numpy(), w)


def test_deterministic(small):
    x = small.x(100, row0=1)
    a = run_forward(small, x, obsmoe.PATH_PREFILL)
    b = run_forward(small, x, obsmoe.PATH_PREFILL)
    c = run_forward(small, x[:3], obsmoe.PATH_DECODE)
    d = run_forward(small, x[:3], obsmoe.PATH_DECODE)
    assert np.array_equal(a, b) and np.array_equal(c, d)


def test_errors(small):
    torch = small.torch
    x = torch.zeros((300, 2048), dtype=torch.int16, device="cuda")
    with pytest.raises(obsmoe.ObsError, match="T out of range"):
        small.ctx.moe_forward(0, x, x, 300)
    with pytest.raises(obsmoe.ObsError, match="layer"):
        small.ctx.moe_forward(7, x, x, 1)
    shape = obsmoe.MoeShape(2048, 256, 16, 4, n_layers=1, max_tokens=8)
    ctx = obsmoe.MoeContext(shape, 0)
    with pytest.raises(obsmoe.ObsError, match="not loaded"):
        ctx.moe_forward(0, x, x, 1)
    ctx.close()


@pytest.mark.parametrize("path,T,launches", [(obsmoe.PATH_PREFILL, 100, 3), (obsmoe.PATH_DECODE, 3, 1),
                                            (obsmoe.PATH_DECODE, 8, 1), (obsmoe.PATH_DECODE, 12, 3)])
def test_forward_replays_from_a_cuda_graph(small, path, T, launches):
    """The layer forward issues only stream-ordered work, so it can be captured
    in a CUDA graph (the fused decode layer of T <= 8 is one cooperative launch);
    replays give the eager result bit for bit."""
    torch = small.torch
    x = dev(torch, small.x(T, row0=21))
    eager = torch.empty((T, 2048), dtype=torch.int16, device="cuda")
    n0 = obsmoe.kernel_launches()
    small.ctx.moe_forward(0, x, eager, T, path=path)
    per_forward = obsmoe.kernel_launches() - n0
    assert per_forward >= launches
    out = torch.full((T, 2048), -1, dtype=torch.int16, device="cuda")
    cap = torch.cuda.Stream()
    cap.wait_stream(torch.cuda.current_stream())
    g = torch.cuda.CUDAGraph()
    with torch.cuda.stream(cap):
        with torch.cuda.graph(g, stream=cap):
            small.ctx.moe_forward(0, x, out, T, path=path, stream=cap)
    torch.cuda.current_stream().wait_stream(cap)
    for _ in range(2):
        out.fill_(-1)
        g.replay()
        torch.cuda.synchronize()
        assert torch.equal(out, eager)
    del g
    small.ctx.check_device()


def test_rmsnorm_bit_exact(small):
    """The stack's layer-input norm: bit-exact with the oracle (rmsnorm.metal's order)."""
    torch = small.torch
    x = O.f32_to_bf16(O.bf16_to_f32(small.x(33, row0=7)) * np.float32(2.5) + np.float32(0.1))
    out = torch.empty((33, 2048), dtype=torch.int16, device="cuda")
    small.ctx.rmsnorm(dev(torch, x), out, 33)
    assert np.array_equal(host(out, np.uint16), O.rmsnorm_layer(x))


@pytest.mark.parametrize("T,path", [(40, obsmoe.PATH_PREFILL), (3, obsmoe.PATH_DECODE)])
def test_layer_stack(cuda, T, path):
    """Three layers on a residual stream: the stack entry equals the per-layer calls
    bit for bit, and the oracle chain within tolerance."""
    torch = cuda
    n = 3
    shape = obsmoe.MoeShape(2048, 256, 16, 4, n_layers=n, max_tokens=64)
    ctx = obsmoe.MoeContext(shape, 0)
    Ls = [O.synth_layer(9, l, E=16, H=2048, I=256, K=4) for l in range(n)]
    for l, L in enumerate(Ls):
        ctx.load_layer(l, L)
    r0 = small_resid = O.synth_x(9, 5, T, 2048)
    r = dev(torch, r0)
    ctx.moe_stack_forward(0, n, r, T, path=path)
    got = host(r, np.uint16)
    # the same chain through the single-layer entry points
    m = dev(torch, small_resid)
    xn = torch.empty_like(m)
    nxt = torch.empty_like(m)
    for l in range(n):
        ctx.rmsnorm(m, xn, T)
        ctx.moe_forward(l, xn, nxt, T, residual=m, path=path)
        m, nxt = nxt, m
    assert np.array_equal(got, host(m, np.uint16))
    ref = O.moe_stack(Ls, r0, wmode=1 if path == obsmoe.PATH_PREFILL else 0)
    assert rel_err(O.bf16_to_f32(got), O.bf16_to_f32(ref)) < REL
    ctx.check_device()
    ctx.close()
