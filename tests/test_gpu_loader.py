"""Layers loaded from the reference splitter's expert files (obs_load_layer_safetensors)
against the same layers loaded from arrays: identical HBM contents, so identical
forwards bit for bit, on the small shape and on the full Qwen3-30B-A3B shape."""
import numpy as np
import pytest

import obsmoe
import oracle as O
from expert_files import write_layer_file
from parity_util import REL, dev, host, rel_err

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("E,I,K", [(16, 256, 4), (128, 768, 8)])
def test_file_loaded_layer_equals_array_loaded(cuda, tmp_path, E, I, K):
    torch = cuda
    H = 2048
    L = O.synth_layer(12, 0, E=E, H=H, I=I, K=K)
    path = write_layer_file(tmp_path / "layer_0_experts.safetensors", L)
    assert obsmoe.expert_file_info(str(path)) == (E, H, I)
    shape = obsmoe.MoeShape(H, I, E, K, n_layers=1, max_tokens=128)
    a = obsmoe.MoeContext(shape, 0)
    a.load_layer(0, L)
    b = obsmoe.MoeContext(shape, 0)
    b.load_layer_file(0, str(path), L.router_w, L.router_s, L.router_b)
    for T, path_ in ((1, obsmoe.PATH_DECODE), (100, obsmoe.PATH_PREFILL)):
        xh = O.synth_x(12, 0, T, H, row0=5)
        x = dev(torch, xh)
        outs = []
        for ctx in (a, b):
            out = torch.empty((T, H), dtype=torch.int16, device="cuda")
            ctx.moe_forward(0, x, out, T, path=path_)
            torch.cuda.synchronize()
            outs.append(host(out, np.uint16).copy())
        assert np.array_equal(outs[0], outs[1]), (T, path_)
        ref, _, _ = O.moe_layer(L, xh, wmode=0)
        assert rel_err(outs[1], ref) < REL
    # a file of another shape is refused with a message
    if E == 16:
        small = O.synth_layer(12, 0, E=8, H=H, I=I, K=K)
        p2 = write_layer_file(tmp_path / "other.safetensors", small)
        with pytest.raises(obsmoe.ObsError, match="differs from the context"):
            b.load_layer_file(0, str(p2), small.router_w, small.router_s, small.router_b)
    a.check_device()
    b.check_device()
    a.close()
    b.close()
