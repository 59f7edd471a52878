"""Seeded synthetic inputs of the BASELINE workloads that are not weights or
activations (those come from the library's own generator, obs_synth_layer /
obs_synth_activations): config 3's skewed expert load.

Config 3 adds a Zipf(s = 1.1) per-expert bias to the router logits so the
expert load is skewed: bias_e = beta * log(r_e ** -1.1), r a seeded rank
permutation of the experts (r = 1 the hottest).  The reference's router has no
such input (shaders/dequant_matvec_8bit.metal:8-31); it enters through
obs_moe_forward's logit_bias.  beta = 4.9 puts the hottest expert at 9.98x the
mean load on layer 0 of seed 0 at T = 4096 (2,554 of 32,768 routed rows)."""
from __future__ import annotations

import numpy as np

CONFIG3_BETA = 4.9
ZIPF_S = 1.1


def zipf_bias(beta: float, n_experts: int = 128, seed: int = 11) -> np.ndarray:
    """fp32 [n_experts] logit bias beta * log(r_e ** -s) over a seeded rank permutation."""
    r = np.random.default_rng(seed).permutation(n_experts) + 1
    return (beta * -ZIPF_S * np.log(r)).astype(np.float32)
