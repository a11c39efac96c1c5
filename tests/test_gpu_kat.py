"""The trained-weight known answer, on the device.

The reference's own trained checkpoints (artifacts/target.pt: d_model 128,
4 layers, SwiGLU 352; artifacts/draft.pt: d_model 64, 2 layers, SwiGLU 160;
both float32, vocab 65) and the eight 32-token prompts of the reference's
scripts/verify_speculative.py:236-241 (seed 20240) are stored as arrays by
``tests/golden/make_golden.py``, which also ran the reference on them.  For
gamma 1/2/4/7 the speculative greedy output of every prompt (48 tokens)
must equal the dense greedy continuation, per-prompt acceptance counts must
equal the reference's, and the acceptance rate of the last prompt (the
figure the reference publishes, artifacts/spec_stats.json:6-35, because
its script resets the decoder before each prompt) must be 0.7142857 /
0.6428571 / 0.4558824 / 0.3469388.
"""

from __future__ import annotations

from pathlib import Path

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

KAT = Path(__file__).resolve().parent / "golden" / "kat_fixtures.npz"
PUBLISHED = {1: 0.7142857142857143, 2: 0.6428571428571429, 4: 0.45588235294117646,
             7: 0.3469387755102041}


@pytest.fixture(scope="module")
def kat() -> dict[str, np.ndarray]:
    with np.load(KAT) as z:
        return {k: z[k] for k in z.files}


def _model(kat, which: str):
    from microserve_b200.config import ModelConfig
    from microserve_b200.model import Transformer

    v, L, d, h, hkv, ff, msl = (int(x) for x in kat[f"{which}_cfg"])
    cfg = ModelConfig(vocab_size=v, n_layers=L, d_model=d, n_heads=h, n_kv_heads=hkv, d_ff=ff,
                      max_seq_len=msl)
    pre = which + "/"
    st = {k[len(pre):]: a for k, a in kat.items() if k.startswith(pre)}
    st["lm_head.weight"] = st["embed.weight"]
    return Transformer.from_state_dict(cfg, st, "cuda")


@pytest.mark.parametrize("gamma", [1, 2, 4, 7])
def test_trained_checkpoints_reproduce_the_published_acceptance(kat, gamma: int) -> None:
    from microserve_b200.config import CacheConfig, SamplingConfig
    from microserve_b200.speculative import SpeculativeDecoder

    target, draft = _model(kat, "target"), _model(kat, "draft")
    dec = SpeculativeDecoder(target, draft, CacheConfig(block_size=16, num_blocks=256),
                             gamma=gamma)
    counts = []
    matches = 0
    for i, prompt in enumerate(kat["prompts"].tolist()):
        dec.reset()
        got = dec.generate(prompt, SamplingConfig(temperature=0.0, max_new_tokens=48), seq_id=i)
        assert got == kat[f"spec{gamma}/{i}"].tolist(), f"prompt {i}"
        matches += int(got == kat["dense"][i].tolist())
        counts.append([dec.num_accepted, dec.num_proposed])
    assert matches == 8
    assert counts == kat[f"spec{gamma}/counts"].tolist()
    assert counts[-1][0] / counts[-1][1] == pytest.approx(PUBLISHED[gamma], abs=1e-12)
