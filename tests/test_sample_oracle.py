"""The oracle's sampling restatement (src/main.rs:192-305) against an
independent f32 restatement in Python on small vocabularies.  The reference
ships no sampling tests or fixtures, so this pins the C code to a second
reading of the same lines: penalty per distinct recent id, temperature,
softmax with sequential sums, top-p over p > 1e-5 sorted descending (ties to
the lower id), the r -= p walk."""
import numpy as np
import pytest

f32 = np.float32


def py_sample(logits, recent, penalty, temperature, top_p, u):
    l = [f32(x) for x in logits]
    V = len(l)
    if penalty > 1.0:
        seen = set()
        for id_ in recent:
            if id_ in seen or not (0 <= id_ < V):
                continue
            seen.add(id_)
            s = l[id_]
            l[id_] = f32(s * f32(penalty)) if s < 0 else f32(s / f32(penalty))
    if abs(f32(temperature) - f32(1.0)) > f32(1e-6):
        l = [f32(x / f32(temperature)) for x in l]
    mx = f32(-3.4028235e38)
    for x in l:
        mx = max(mx, x)
    p = [f32(np.exp(f32(x - mx))) for x in l]
    s = f32(0.0)
    for x in p:
        s = f32(s + x)
    p = [f32(x / s) for x in p]
    if top_p < 1.0:
        c = [(x, i) for i, x in enumerate(p) if x > f32(1e-5)] or [(x, i) for i, x in enumerate(p)]
        c.sort(key=lambda t: (-t[0], t[1]))
        cum, cut = f32(0.0), len(c) - 1
        for i, (x, _) in enumerate(c):
            cum = f32(cum + x)
            if cum > f32(top_p):
                cut = i
                break
        total = f32(0.0)
        for x, _ in c[:cut + 1]:
            total = f32(total + x)
        r = f32(f32(u) * total)
        for x, i in c[:cut + 1]:
            r = f32(r - x)
            if r <= 0:
                return i
        return c[0][1]
    r = f32(u)
    for i, x in enumerate(p):
        r = f32(r - x)
        if r <= 0:
            return i
    return 0


@pytest.mark.parametrize("sigma,penalty,temperature,top_p", [(3.0, 1.3, 0.8, 0.9), (0.05, 1.0, 1.0, 0.5),
                                                             (2.0, 1.1, 1.0, 1.0), (8.0, 1.5, 1.7, 0.95)])
def test_oracle_sample_matches_python_restatement(orc, sigma, penalty, temperature, top_p):
    rng = np.random.default_rng(int(sigma * 100) + int(top_p * 10))
    V = 700
    for trial in range(6):
        logits = rng.normal(0, sigma, V).astype(np.float32)
        recent = rng.integers(0, V, 40).tolist() + [3, 3, 5]
        u = float(rng.random(dtype=np.float32))
        t_orc, margin = orc.sample(logits, recent, penalty, temperature, top_p, u)
        t_py = py_sample(logits.tolist(), recent, penalty, temperature, top_p, u)
        # the C oracle uses libm expf, numpy its own exp: equal tokens unless the draw sits on a boundary
        assert t_orc == t_py or margin < 1e-6, (trial, t_orc, t_py, margin)
