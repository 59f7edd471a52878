"""BASELINE configs 2 and 3 at full shape (E=128, I=768, K=8, H=2048) through
the C ABI against the oracle.

* Config 3: one layer of the T=4096 prefill with the Zipf(1.1) logit bias (the
  hottest expert gets ~2,550 of 32,768 routed rows, about 40 token tiles of one
  expert).  Every token's expert ids are checked bit for bit; outputs of a
  token sample (random rows plus the tail rows, which land in the last tiles of
  the hot experts' segments) against the oracle; and at the full size, a
  size-independent property: a token permutation of the batch permutes the
  outputs bit for bit (each token's result is independent of which tile or
  which neighbours it was computed with).
* Config 2: one layer at B = 8, 32 and 128 decode tokens, every path.
* The layer stack: two full-shape layers on a residual stream.
"""
import numpy as np
import pytest

import obsmoe
import oracle as O
import synthetic
from parity_util import REL, REL_ELEM, REL_SAME, dev, elem_err, host, rel_err

pytestmark = pytest.mark.gpu

E, H, I, K = 128, 2048, 768, 8
T3 = 4096
DECODE_MAX = 8


@pytest.fixture(scope="module")
def cfg3(cuda):
    torch = cuda
    ctx = obsmoe.MoeContext(obsmoe.MoeShape(H, I, E, K, n_layers=1, max_tokens=T3), 0)
    L = O.synth_layer(0, 0)
    ctx.load_layer(0, L)
    r0 = O.synth_x(0, 0, T3, H)          # rank 0's residual stream, layer 0 (bench.py's input)
    bias = synthetic.zipf_bias(synthetic.CONFIG3_BETA)
    yield torch, ctx, L, r0, bias
    ctx.check_device()
    ctx.close()


def stack_forward(torch, ctx, r0, T, bias, path, layer0=0, n_layers=1):
    r = dev(torch, r0)
    ctx.moe_stack_forward(layer0, n_layers, r, T, bias=None if bias is None else dev(torch, bias), path=path)
    torch.cuda.synchronize()
    return host(r, np.uint16).copy()


def test_config3_routing_bit_exact_and_skewed(cfg3):
    torch, ctx, L, r0, bias = cfg3
    xn = torch.empty((T3, H), dtype=torch.int16, device="cuda")
    ctx.rmsnorm(dev(torch, r0), xn, T3)
    logits = torch.empty((T3, E), dtype=torch.float32, device="cuda")
    ids = torch.empty((T3, K), dtype=torch.int32, device="cuda")
    wts = torch.empty((T3, K), dtype=torch.float32, device="cuda")
    ctx.gate_gpu(0, xn, logits, T3)
    ctx.route(logits, T3, ids, wts, bias=dev(torch, bias))
    xh = O.rmsnorm_layer(r0)
    assert np.array_equal(host(xn, np.uint16), xh)
    ref_logits = O.router_logits(L, xh)
    assert np.array_equal(host(logits, np.float32).view(np.uint32), ref_logits.view(np.uint32))
    rid, rw = O.topk(ref_logits, K, bias=bias)
    gid = host(ids, np.int32)
    assert np.array_equal(gid, rid)
    assert np.allclose(host(wts, np.float32), rw, rtol=1e-5, atol=1e-7)
    load = np.bincount(gid.ravel(), minlength=E)
    assert 9.0 <= load.max() / load.mean() <= 11.0, load.max() / load.mean()


def test_config3_layer_vs_oracle(cfg3):
    torch, ctx, L, r0, bias = cfg3
    got = stack_forward(torch, ctx, r0, T3, bias, obsmoe.PATH_PREFILL)
    rows = np.unique(np.concatenate([np.random.default_rng(3).choice(T3, 224, replace=False),
                                     np.arange(T3 - 32, T3)]))
    same = O.moe_stack([L], r0[rows], bias=bias, wmode=1)   # the GEMM path's weight arithmetic
    ref = O.moe_stack([L], r0[rows], bias=bias, wmode=0)    # the reference's fp32 weights
    g = got[rows]
    print(f"config 3 sample: normwise {rel_err(g, ref):.2e} (fp32 weights), {rel_err(g, same):.2e} "
          f"(bf16 weights); elementwise {elem_err(g, same):.2e}")
    assert rel_err(g, ref) < REL
    assert rel_err(g, same) < REL_SAME
    assert elem_err(g, same) < REL_ELEM


def test_config3_token_permutation_is_bit_exact(cfg3):
    torch, ctx, L, r0, bias = cfg3
    base = stack_forward(torch, ctx, r0, T3, bias, obsmoe.PATH_PREFILL)
    perm = np.random.default_rng(9).permutation(T3)
    got = stack_forward(torch, ctx, r0[perm], T3, bias, obsmoe.PATH_PREFILL)
    assert np.array_equal(got, base[perm])


@pytest.fixture(scope="module")
def cfg2(cuda):
    torch = cuda
    # OBS_PATH_AUTO takes the decode mat-vec up to DECODE_MAX tokens and the grouped GEMM above
    ctx = obsmoe.MoeContext(obsmoe.MoeShape(H, I, E, K, n_layers=2, max_tokens=128, decode_max_tokens=DECODE_MAX), 0)
    Ls = [O.synth_layer(0, l) for l in range(2)]
    for l, L in enumerate(Ls):
        ctx.load_layer(l, L)
    yield torch, ctx, Ls
    ctx.check_device()
    ctx.close()


@pytest.mark.parametrize("B", [8, 32, 128])
def test_config2_batched_decode_vs_oracle(cfg2, B):
    """One layer of the 48-layer decode stack at batch B, on every path that takes B."""
    torch, ctx, Ls = cfg2
    r0 = O.synth_x(0, 0, B, H)
    paths = [obsmoe.PATH_AUTO, obsmoe.PATH_PREFILL] + ([obsmoe.PATH_DECODE] if B <= 64 else [])
    ref0 = O.moe_stack(Ls[:1], r0, wmode=0)
    ref1 = O.moe_stack(Ls[:1], r0, wmode=1)
    for path in paths:
        got = stack_forward(torch, ctx, r0, B, None, path)
        # the decode mat-vec keeps fp32 weights (wmode 0), the grouped GEMM rounds them to bf16 (wmode 1)
        gemm = path == obsmoe.PATH_PREFILL or (path == obsmoe.PATH_AUTO and B > DECODE_MAX)
        same = ref1 if gemm else ref0
        print(f"B={B} path={path}: normwise {rel_err(got, ref0):.2e}, same-arithmetic {rel_err(got, same):.2e}, "
              f"elementwise {elem_err(got, same):.2e}")
        assert rel_err(got, ref0) < REL
        assert rel_err(got, same) < REL_SAME
        assert elem_err(got, same) < REL_ELEM


@pytest.mark.parametrize("T,path", [(1, obsmoe.PATH_AUTO), (4, obsmoe.PATH_DECODE), (8, obsmoe.PATH_AUTO),
                                    (12, obsmoe.PATH_AUTO), (100, obsmoe.PATH_PREFILL)])
def test_stack_two_full_layers_vs_oracle(cfg2, T, path):
    torch, ctx, Ls = cfg2
    r0 = O.synth_x(0, 7, T, H)
    got = stack_forward(torch, ctx, r0, T, None, path, n_layers=2)
    gemm = path == obsmoe.PATH_PREFILL or (path == obsmoe.PATH_AUTO and T > DECODE_MAX)
    same = O.moe_stack(Ls, r0, wmode=1 if gemm else 0)
    ref = O.moe_stack(Ls, r0, wmode=0)
    print(f"stack T={T} path={path}: normwise {rel_err(got, ref):.2e}, same-arithmetic {rel_err(got, same):.2e}")
    assert rel_err(got, ref) < REL
    # the second layer's input carries the first layer's rounding differences: the per-layer bound twice
    assert rel_err(got, same) < 2 * REL_SAME
