"""The fused decode layer (one cooperative launch for T <= 8) against the
separate decode kernels (router, top-k, gate/up mat-vec, down mat-vec, combine
as separate launches, taken for T = 9).  Every output row depends on its own input
row only, so rows [r, r+T) of a fused call on x[r:r+T] must equal the same rows
of the separate kernels' call on all of x, bit for bit: same router order, same
split-K chains, same combine order.  Also checked against the oracle."""
import numpy as np
import pytest

import obsmoe
import oracle as O

pytestmark = pytest.mark.gpu

REL = 1e-2  # FFN / combine against the oracle: max |gpu - oracle| <= REL * max |oracle|


def dev(torch, a):
    a = np.ascontiguousarray(a)
    view = {np.uint16: np.int16, np.uint32: np.int32}.get(a.dtype.type, a.dtype)
    return torch.from_numpy(a.view(view)).cuda()


def forward(torch, ctx, x, res, bias, T):
    out = torch.full((T, x.shape[1]), -1, dtype=torch.int16, device="cuda")
    ctx.moe_forward(0, x, out, T, residual=res, bias=bias, path=obsmoe.PATH_DECODE)
    torch.cuda.synchronize()
    return out.cpu().numpy().view(np.uint16).copy()


@pytest.mark.parametrize("E,I,K,seed", [(16, 256, 4, 17), (128, 768, 8, 0)])
def test_fused_decode_equals_separate_kernels(cuda, E, I, K, seed):
    torch = cuda
    H, N = 2048, 9
    L = O.synth_layer(seed, 0, E=E, H=H, I=I, K=K)
    ctx = obsmoe.MoeContext(obsmoe.MoeShape(H, I, E, K, n_layers=1, max_tokens=16), 0)
    ctx.load_layer(0, L)
    xn = O.synth_x(seed, 0, N, H, row0=40)
    rn = O.synth_x(seed + 1, 0, N, H, row0=40)
    bias = np.zeros(E, np.float32)
    bias[3] = 0.75
    x, r, b = dev(torch, xn), dev(torch, rn), dev(torch, bias)
    for with_res in (False, True):
        ref = forward(torch, ctx, x, r if with_res else None, b, N)  # T = 9: separate kernels
        for T in (1, 2, 3, 4, 8):
            for r0 in sorted({0, N - T}):
                got = forward(torch, ctx, x[r0:r0 + T], r[r0:r0 + T] if with_res else None, b, T)
                assert np.array_equal(got, ref[r0:r0 + T]), (T, r0, with_res)
        want, _, _ = O.moe_layer(L, xn, bias=bias, residual=rn if with_res else None, wmode=0)
        err = np.abs(O.bf16_to_f32(ref) - O.bf16_to_f32(want)).max() / np.abs(O.bf16_to_f32(want)).max()
        assert err < REL
    ctx.check_device()
    ctx.close()
