"""obs_decode_ffn_static: the decode expert FFN for callers that cannot
allocate device memory (during CUDA graph capture, inside a framework that
owns all device memory, in loops that cannot afford an allocation's implicit
synchronisation).  Its scratch is a fixed array inside the library, so it needs
no context.  Checked through the C ABI against the context's decode path on the
same routes, on two calls in a row; this file runs last in the suite and also
passes on its own in a fresh process."""
import numpy as np
import pytest

import obsmoe
import oracle as O

pytestmark = pytest.mark.gpu

REL = 1e-2  # max |new - existing| <= REL * max |existing|, the suite's FFN tolerance


def dev(torch, a):
    a = np.ascontiguousarray(a)
    view = {np.uint16: np.int16, np.uint32: np.int32}.get(a.dtype.type, a.dtype)
    return torch.from_numpy(a.view(view)).cuda()


class DevWeights:
    """Expert weights of one layer on the device, in the reference (MLX) layout."""

    def __init__(self, torch, L):
        for n in ("gate_w", "gate_s", "gate_b", "up_w", "up_s", "up_b", "down_w", "down_s", "down_b"):
            setattr(self, n, dev(torch, getattr(L, n)))


def test_decode_ffn_static_matches_context_path(cuda):
    torch = cuda
    E, H, I, K, T = 16, 2048, 256, 4, 6
    L = O.synth_layer(31, 0, E=E, H=H, I=I, K=K)
    ctx = obsmoe.MoeContext(obsmoe.MoeShape(H, I, E, K, n_layers=1, max_tokens=16), 0)
    ctx.load_layer(0, L)
    w = DevWeights(torch, L)
    for call in range(2):  # two calls in a row share the library's scratch
        x = dev(torch, O.synth_x(31, 0, T, H, row0=100 * call))
        res = dev(torch, O.synth_x(32, 0, T, H, row0=100 * call)) if call == 1 else None
        # the existing entry point: the context's decode path
        ref = torch.empty((T, H), dtype=torch.int16, device="cuda")
        ctx.moe_forward(0, x, ref, T, residual=res, path=obsmoe.PATH_DECODE)
        # the same routes through the router entry points
        logits = torch.empty((T, E), dtype=torch.float32, device="cuda")
        ids = torch.empty((T, K), dtype=torch.int32, device="cuda")
        wts = torch.empty((T, K), dtype=torch.float32, device="cuda")
        ctx.gate_gpu(0, x, logits, T)
        ctx.route(logits, T, ids, wts)
        out = torch.full((T, H), -1, dtype=torch.int16, device="cuda")
        obsmoe.decode_ffn_static(w, E, H, I, K, x, ids, wts, T, out, residual=res)
        torch.cuda.synchronize()
        a = O.bf16_to_f32(out.cpu().numpy().view(np.uint16))
        b = O.bf16_to_f32(ref.cpu().numpy().view(np.uint16))
        assert np.abs(a - b).max() <= REL * np.abs(b).max(), f"call {call}"
    ctx.check_device()
    ctx.close()


def test_decode_ffn_static_rejects_oversize(cuda):
    torch = cuda
    E, H, I, K = 16, 2048, 256, 4
    L = O.synth_layer(31, 0, E=E, H=H, I=I, K=K)
    w = DevWeights(torch, L)
    T = 17  # T * K = 68 > OBS_STATIC_MAX_PAIRS
    x = torch.zeros((T, H), dtype=torch.int16, device="cuda")
    ids = torch.zeros((T, K), dtype=torch.int32, device="cuda")
    wts = torch.zeros((T, K), dtype=torch.float32, device="cuda")
    with pytest.raises(obsmoe.ObsError, match="OBS_STATIC_MAX_PAIRS"):
        obsmoe.decode_ffn_static(w, E, H, I, K, x, ids, wts, T, x)
    with pytest.raises(obsmoe.ObsError, match="inter"):
        obsmoe.decode_ffn_static(w, E, H, 4096, K, x[:2], ids[:2], wts[:2], 2, x[:2])
