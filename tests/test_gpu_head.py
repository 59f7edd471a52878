"""The model's ends on the GPU against the oracle at the full Qwen3-30B-A3B shape
(vocabulary 151,936, H 2048): the embedding rows bit for bit; the final RMSNorm +
lm_head logits bit for bit (one canonical fp32 order) and therefore the greedy
next tokens, for one token and for a batch of 16."""
import numpy as np
import pytest

import obsmoe
import oracle as O
from parity_util import dev, host

pytestmark = pytest.mark.gpu

VOCAB, H = 151936, 2048


@pytest.fixture(scope="module")
def head(cuda):
    hd = O.synth_head(0, vocab=VOCAB, H=H)
    ctx = obsmoe.MoeContext(obsmoe.MoeShape(H, 768, 128, 8, n_layers=1, max_tokens=16), 0)
    ctx.load_head(VOCAB, hd)
    yield cuda, ctx, hd
    ctx.check_device()
    ctx.close()


def test_embed_rows_bit_exact(head):
    torch, ctx, hd = head
    toks = np.array([0, 1, 9707, 271, VOCAB - 1, 151643, 77, 9707], np.int32)
    x = torch.empty((len(toks), H), dtype=torch.int16, device="cuda")
    ctx.embed(dev(torch, toks), len(toks), x)
    torch.cuda.synchronize()
    assert np.array_equal(host(x, np.uint16), O.embed(hd, toks))


@pytest.mark.parametrize("T", [1, 16])
def test_lm_head_logits_and_next_tokens_bit_exact(head, T):
    torch, ctx, hd = head
    # a residual stream as the last layer leaves it: synthetic rows scaled off unit rms
    xh = O.f32_to_bf16(O.bf16_to_f32(O.synth_x(5, 47, T, H)) * np.float32(3.5))
    ids = torch.empty(T, dtype=torch.int32, device="cuda")
    logits = torch.empty((T, VOCAB), dtype=torch.float32, device="cuda")
    ctx.lm_head(dev(torch, xh), T, ids, logits)
    torch.cuda.synchronize()
    ref_logits, ref_ids = O.lm_head(hd, xh)
    assert np.array_equal(host(logits, np.float32).view(np.uint32), ref_logits.view(np.uint32))
    assert np.array_equal(host(ids, np.int32), ref_ids)
    # without a logits buffer the ids are the same
    ids2 = torch.empty(T, dtype=torch.int32, device="cuda")
    ctx.lm_head(dev(torch, xh), T, ids2)
    torch.cuda.synchronize()
    assert torch.equal(ids, ids2)


def test_head_errors(head):
    torch, ctx, hd = head
    x = torch.zeros((17, H), dtype=torch.int16, device="cuda")
    ids = torch.empty(17, dtype=torch.int32, device="cuda")
    with pytest.raises(obsmoe.ObsError, match="T out of range"):
        ctx.lm_head(x, 17, ids)
    c2 = obsmoe.MoeContext(obsmoe.MoeShape(H, 768, 128, 8, n_layers=1, max_tokens=4), 0)
    with pytest.raises(obsmoe.ObsError, match="head not loaded"):
        c2.lm_head(x, 1, ids)
    c2.close()
