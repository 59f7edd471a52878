"""Failure detection on the GPU without a GPU fault: every device-side wait of
the library is bounded, and a wait that runs out records a timeout that the
host reads as OBS_ERR_TIMEOUT while the context stays usable.

The wait is made to run out on purpose with obs_probe_wait: one wait, the
expert-parallel receive's own device code, on a stamp that nothing writes,
under a 10 ms limit.  The reference's failure paths are host-side only
(src/forward.rs:190,432,498-507)."""
import time

import pytest

import obsmoe
import oracle as O
from parity_util import dev

pytestmark = pytest.mark.gpu


def test_bounded_wait_runs_out_and_context_survives(cuda):
    torch = cuda
    E, H, I, K, T = 16, 2048, 256, 4, 24
    ctx = obsmoe.MoeContext(obsmoe.MoeShape(H, I, E, K, n_layers=1, max_tokens=64), 0)
    ctx.load_layer(0, O.synth_layer(4, 0, E=E, H=H, I=I, K=K))
    x = dev(torch, O.synth_x(4, 0, T, H))
    want = torch.empty((T, H), dtype=torch.int16, device="cuda")
    ctx.moe_forward(0, x, want, T, path=obsmoe.PATH_PREFILL)
    ctx.check_device()

    ctx.set_wait_limit(10_000_000)  # 10 ms
    t0 = time.perf_counter()
    ctx.probe_wait()
    with pytest.raises(obsmoe.ObsError) as ei:
        ctx.check_device()
    dt = time.perf_counter() - t0
    assert ei.value.status == 5 and "gave up" in str(ei.value)   # OBS_ERR_TIMEOUT
    assert 0.01 <= dt < 1.5, dt                                    # the limit, not the 2 s default
    ctx.check_device()                                             # the flag is cleared

    # the context and the GPU keep working: the same forward, bit for bit, under the short limit
    got = torch.full((T, H), -1, dtype=torch.int16, device="cuda")
    ctx.moe_forward(0, x, got, T, path=obsmoe.PATH_PREFILL)
    ctx.check_device()
    assert torch.equal(got, want)
    for path, Tp in ((obsmoe.PATH_DECODE, 2), (obsmoe.PATH_DECODE, 7)):
        a = torch.empty((Tp, H), dtype=torch.int16, device="cuda")
        ctx.moe_forward(0, x[:Tp], a, Tp, path=path)
        ctx.check_device()

    ctx.set_wait_limit(0)  # back to the default
    with pytest.raises(obsmoe.ObsError, match="wait limit"):
        ctx.set_wait_limit(1000)  # below 1 ms
    ctx.close()
