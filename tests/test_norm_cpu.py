"""The oracle's norm + residual restatement (oracle.rms_residual) against a
pure-Python loop of the same steps on a tiny case (float32 arithmetic, bf16
storage between the steps), so the GPU test's reference is itself checked."""
import math

import numpy as np

from oracle import oracle as O


def _bf(v: float) -> float:
    return float(O.bf16_to_f64(O.f32_to_bf16(np.array([v], dtype=np.float32)))[0])


def _loop(x, o, og, gate, ng, eps):
    m, h = x.shape
    xs = [[float(v) for v in row] for row in O.bf16_to_f64(x)]
    og = [float(v) for v in O.bf16_to_f64(og)]
    ng = [float(v) for v in O.bf16_to_f64(ng)]
    gate = [math.tanh(float(v)) for v in O.bf16_to_f64(gate)]
    os_ = O.bf16_to_f64(o)
    nrm = []
    for r in range(m):
        ov = [float(v) for v in os_[r]]
        ro = 1.0 / math.sqrt(sum(v * v for v in ov) / h + eps)
        s = [_bf(ov[i] * ro * og[i]) for i in range(h)]
        xs[r] = [_bf(xs[r][i] + gate[i] * s[i]) for i in range(h)]
        rx = 1.0 / math.sqrt(sum(v * v for v in xs[r]) / h + eps)
        nrm.append([_bf(xs[r][i] * rx * ng[i]) for i in range(h)])
    return np.array(xs), np.array(nrm)


def test_oracle_rms_residual_matches_loop():
    rng = np.random.default_rng(0)
    m, h = 5, 64
    bits = lambda a: O.f32_to_bf16(np.asarray(a, dtype=np.float32))  # noqa: E731
    x, o = bits(rng.normal(size=(m, h))), bits(rng.normal(size=(m, h)) * 2)
    og, ng = bits(rng.uniform(0.5, 1.5, h)), bits(rng.uniform(0.5, 1.5, h))
    gate = bits(rng.normal(size=h))
    xr, nr = O.rms_residual(x, o, og, gate, ng, 1e-5)
    xl, nl = _loop(x, o, og, gate, ng, 1e-5)
    # float32 vs float64 intermediate math: equal up to rare bf16 rounding ties
    assert O.rel_l2(O.bf16_to_f64(xr), xl) < 1e-3
    assert O.rel_l2(O.bf16_to_f64(nr), nl) < 1e-3
    assert np.mean(O.bf16_to_f64(xr) != xl) < 0.03
