"""Error metrics and device plumbing shared by the GPU parity tests.

Two error measures of a bf16 output against the oracle:
* normwise: max_i |got_i - ref_i| / max_i |ref_i|.  The north star's contract
  (max relative error 1e-2 in bf16) is asserted in this form.
* elementwise: max_i |got_i - ref_i| / max(|ref_i|, floor), floor = rms(ref).
  Outputs are sums of eight weighted expert rows (plus the residual), so some
  cancel to near zero; an element smaller than a typical output is compared on
  the scale of a typical output.  Against the oracle run in the same weight
  arithmetic, the two sides differ only in fp32 accumulation order, which moves
  a bf16 intermediate (h, y) or the output by about one bf16 ulp (2^-8 .. 2^-7
  relative): the bound is 2e-2.  (With a floor of 0.1 * rms the same runs
  measure 2.5e-2 .. 5.5e-2: one ulp of a typical output over a tenth of it.)"""
from __future__ import annotations

import numpy as np

import oracle as O

REL = 1e-2          # normwise, against the oracle (north star)
REL_SAME = 5e-3     # normwise, against the oracle run in the same weight arithmetic
ELEM_FLOOR = 1.0    # elementwise floor, as a fraction of rms(ref)
REL_ELEM = 2e-2     # elementwise, against the oracle run in the same weight arithmetic


def as_f32(a):
    a = np.asarray(a)
    return O.bf16_to_f32(a) if a.dtype == np.uint16 else a.astype(np.float32)


def rel_err(got, ref) -> float:
    got, ref = as_f32(got), as_f32(ref)
    return float(np.abs(got - ref).max() / max(float(np.abs(ref).max()), 1e-30))


def elem_err(got, ref, floor: float = ELEM_FLOOR) -> float:
    got, ref = as_f32(got), as_f32(ref)
    rms = float(np.sqrt(np.mean(ref.astype(np.float64) ** 2)))
    return float((np.abs(got - ref) / np.maximum(np.abs(ref), floor * rms)).max())


def dev(torch, a):
    a = np.ascontiguousarray(a)
    view = {np.uint16: np.int16, np.uint32: np.int32}.get(a.dtype.type, a.dtype)
    return torch.from_numpy(a.view(view)).cuda()


def host(t, dtype):
    return t.detach().cpu().contiguous().numpy().view(dtype)
