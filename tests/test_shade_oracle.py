"""The shading oracle's BRDF terms against their published closed forms
(test/brdf.test.ts:57-81), on CPU.

The literal float32 evaluation of the reference's GGX formula,
a2 / (pi * (n.h^2 (a2 - 1) + 1)^2), loses ~0.23 % at n.h = 1 and roughness
0.04 to cancellation in (a2 - 1) + 1, so the bound here is 3e-3 rather than
the 1e-3 the reference quotes for its GPU.
"""
import math


def test_ggx_and_smith_closed_forms():
    from oracle import lib
    worst = 0.0
    for r in [0.04, 0.08, 0.12, 0.155, 0.2, 0.3, 0.55, 1.0]:
        for nh in [1.0, 0.9999, 0.999, 0.99, 0.9, 0.7, 0.5]:
            a = r * r
            a2 = a * a
            den = nh * nh * (a2 - 1) + 1
            d_ref = a2 / (math.pi * den * den)
            k = (r + 1) ** 2 / 8
            g_ref = (0.8 / (0.8 * (1 - k) + k)) * (0.6 / (0.6 * (1 - k) + k))
            worst = max(worst, abs(lib().or_ggx_d(nh, r) / d_ref - 1))
            assert abs(lib().or_smith_g(0.8, 0.6, r) - g_ref) < 1e-6
    assert worst < 3e-3
