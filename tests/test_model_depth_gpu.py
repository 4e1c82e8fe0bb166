"""Full-depth greedy parity: the 32-layer 8B W4 and the 16-layer 1B W8 models
(BASELINE configs 3 and 2 at their full layer counts, synthetic seeded
weights) through am_session_generate against the CPU oracle.

Every generated position is compared, not only those before the first
difference: when the engine picks another token than the oracle at position
i, the oracle's top-1/top-2 logit gap there must be a documented near-tie
(below NEAR_TIE), and the engine is restarted on the oracle's own prefix
(prompt + oracle tokens 0..i) to continue the comparison from i + 1. The
number of such near-tie flips is reported and bounded.

NEAR_TIE is 0.125 in logit units: logits are stored in bf16 (the reference
Linear's output dtype), whose spacing is 0.03125 for logits in [4, 8), so the
threshold is 4 bf16 ulps there; engine and oracle sum in different orders in
fp32 over 16-32 layers, which moves a logit by a few ulps.
"""
import dataclasses

import numpy as np
import pytest

from tests.model_fixtures import NEAR_TIE_BF16 as NEAR_TIE, walk_greedy

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("cfg_name,new,seed", [("LLAMA_8B_W4", 16, 0), ("LLAMA_1B_W8", 24, 0)])
def test_full_depth_greedy_matches_oracle(built_lib, oracle_lib, cfg_name, new, seed):
    from aethermind_b200 import session
    base = getattr(session, cfg_name)
    cfg = dataclasses.replace(base, max_seq=128, max_batch=1)
    assert cfg.layers == base.layers  # the named model's full depth
    prompt = np.random.default_rng(100 + seed).integers(0, cfg.vocab, 16).astype(np.uint32)
    om = oracle_lib.synthetic_oracle_model(cfg, seed=seed)
    ref, gaps = om.generate(prompt.astype(np.int64), new)
    del om
    rt = session.Runtime(0)
    m = session.Model(rt, cfg)
    m.init_synthetic(seed=seed)
    s = session.Session(m)
    flips = walk_greedy(s, prompt, ref, gaps, NEAR_TIE)
    near = int((gaps < NEAR_TIE).sum())
    print(f"\n{cfg_name} ({cfg.layers} layers): {new} positions, {near} oracle near-ties (gap < {NEAR_TIE}), "
          f"{len(flips)} flipped at {flips}; oracle gaps {np.round(gaps, 4).tolist()}")
    # a flip needs a near-tie; most positions must match outright
    assert len(flips) <= new // 4, f"{len(flips)} near-tie flips in {new} positions: {flips}"
