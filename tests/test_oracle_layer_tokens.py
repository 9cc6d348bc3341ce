"""The per-token layer oracle (moe_layer_tokens) against the full-layer oracle.

moe_layer_tokens recomputes only the rows of the requested tokens, fetching
each expert's weights once; the full-size GPU layer test relies on it. Here
it must reproduce moe_layer's output for the same tokens (GEMM rows depend
only on their own inputs, so only fp32 summation order inside a dot product
can differ: within one bf16 ulp).
"""
import numpy as np
import pytest

from oracle import moe_oracle as orc


@pytest.mark.parametrize("t,h,e,f,k,zipf", [(96, 256, 16, 128, 4, False),
                                            (200, 512, 32, 256, 8, True)])
def test_tokens_oracle_matches_full_layer(t, h, e, f, k, zipf):
    rng = np.random.default_rng(t + e)
    x = orc.f32_to_bf16(rng.standard_normal((t, h), dtype=np.float32))
    lg = rng.standard_normal((t, e), dtype=np.float32)
    bias = (-1.5 * np.log(rng.permutation(e) + 1.0)).astype(np.float32) if zipf else None
    w1 = orc.f32_to_bf16(rng.standard_normal((e, 2 * f, h), dtype=np.float32) * 0.05)
    w2 = orc.f32_to_bf16(rng.standard_normal((e, h, f), dtype=np.float32) * 0.05)
    ref = orc.moe_layer(x, lg, w1, w2, k, bias)
    _, _, _, probs = orc.router(lg, k, bias)
    toks = np.array([0, t - 1, 3, t // 2, 17])
    fetched = []

    def w1_of(i):
        fetched.append(i)
        return w1[i]

    got = orc.moe_layer_tokens(x, probs, toks, w1_of, lambda i: w2[i])
    assert len(fetched) == len(set(fetched))  # each expert fetched once
    a, b = orc.bf16_to_f32(got), orc.bf16_to_f32(ref[toks])
    ulp = np.abs(b) * 2.0 ** -7 + 1e-30
    assert np.all(np.abs(a - b) <= ulp), np.abs(a - b).max()
