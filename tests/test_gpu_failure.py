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


@pytest.mark.parametrize("case", ["expert", "rows_past_buffer", "rows_unaligned", "rows_above_tile", "count"])
def test_corrupt_gemm_tiles_are_refused(cuda, case):
    """A token-tile list the dispatch could never produce (made on the host and handed
    to the gate/up GEMM through obs_debug_gemm_tiles) is refused by the GEMM's own
    check before any work: kDevBadTile, reported as OBS_ERR_INVALID; the context keeps
    working afterwards."""
    torch = cuda
    E, H, I, K, T = 16, 2048, 256, 4, 64
    ctx = obsmoe.MoeContext(obsmoe.MoeShape(H, I, E, K, n_layers=1, max_tokens=T), 0)
    ctx.load_layer(0, O.synth_layer(4, 0, E=E, H=H, I=I, K=K))
    good = [[0, 0, 16, 0], [3, 16, 32, 0]]
    ctx.debug_gemm_tiles(0, good)
    ctx.check_device()  # a valid list runs
    bad = {"expert": [[E, 0, 16, 0]],
           "rows_past_buffer": [[1, 100000, 16, 0]],
           "rows_unaligned": [[1, 0, 24, 0]],
           "rows_above_tile": [[1, 0, 128, 0]],
           # more tiles than the tile buffer holds (each entry valid on its own)
           "count": [[0, 0, 16, 0]] * 1000}[case]
    ctx.debug_gemm_tiles(0, bad)
    with pytest.raises(obsmoe.ObsError, match="GEMM tile") as ei:
        ctx.check_device()
    assert ei.value.status == 1  # OBS_ERR_INVALID
    x = dev(torch, O.synth_x(4, 0, 8, H))
    a = torch.empty((8, H), dtype=torch.int16, device="cuda")
    b = torch.empty((8, H), dtype=torch.int16, device="cuda")
    ctx.moe_forward(0, x, a, 8, path=obsmoe.PATH_PREFILL)
    ctx.moe_forward(0, x, b, 8, path=obsmoe.PATH_PREFILL)
    ctx.check_device()
    assert torch.equal(a, b)
    ctx.close()
