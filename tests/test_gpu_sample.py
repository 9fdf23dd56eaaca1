"""Device-side sampling (llmrs_sample) against the oracle's restatement of
src/main.rs:192-305, on full-vocabulary logits.  The draw u is shared.

The probabilities agree to rounding (tree sum, CUDA expf), so for peaked
distributions the sampled token must be the oracle's (or the oracle's walk
ended within 1e-6 of a boundary).  For near-uniform distributions the token
is decided by last-bit differences that no reordered sum reproduces: there
the roulette pick must sit at the oracle's cumulative position to within
1e-4 (the walk's accumulated rounding over 128k terms), and the top-p pick
must be one of the oracle's nucleus candidates."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

V = 128256


def probs64(logits, recent, penalty, temperature):
    l = logits.astype(np.float64).copy()
    if penalty > 1.0:
        for i in set(int(x) for x in recent if 0 <= x < len(l)):
            l[i] = l[i] * penalty if l[i] < 0 else l[i] / penalty
    if abs(temperature - 1.0) > 1e-6:
        l /= temperature
    e = np.exp(l - l.max())
    return e / e.sum()


def check(t_gpu, t_orc, margin, p, top_p, u, flat):
    if t_gpu == t_orc or margin < 1e-6:
        return True
    if not flat:
        return False
    if top_p >= 1.0:  # roulette: same cumulative position
        c = np.concatenate([[0.0], np.cumsum(p)])
        return abs(c[t_gpu] - c[t_orc]) < 1e-4
    cand = np.flatnonzero(p > 1e-5)
    if cand.size == 0:
        cand = np.arange(p.size)
    return t_gpu in set(cand.tolist())


@pytest.mark.parametrize("sigma,penalty,temperature,top_p,flat", [
    (6.0, 1.3, 0.7, 0.9, False),   # peaked: a few candidates, sorted in shared memory
    (1.0, 1.1, 1.0, 0.9, False),   # ~30k candidates: sorted in global memory
    (0.01, 1.0, 1.0, 0.9, True),   # flat: no p > 1e-5, every id is a candidate
    (3.0, 1.2, 1.3, 1.0, False),   # roulette over all ids
    (0.5, 1.0, 1.0, 1.0, True),    # flat roulette
])
def test_sample_matches_oracle(llmrs, ctx, be, orc, sigma, penalty, temperature, top_p, flat):
    rng = np.random.default_rng(int(sigma * 1000) + int(top_p * 7))
    for trial in range(4):
        logits = rng.normal(0, sigma, V).astype(np.float32)
        recent = rng.integers(0, V, 64).tolist() + [int(np.argmax(logits))] * 3
        u = float(rng.random(dtype=np.float32))
        d = llmrs.DeviceTensor.from_numpy(ctx, logits)
        t_gpu = be.sample(d, recent, penalty, temperature, top_p, u)
        t_orc, margin = orc.sample(logits, recent, penalty, temperature, top_p, u)
        p = probs64(logits, recent, penalty, temperature)
        assert check(t_gpu, t_orc, margin, p, top_p, u, flat), (trial, t_gpu, t_orc, margin)


def test_sample_rejects_bad_draw(llmrs, ctx, be):
    d = llmrs.DeviceTensor.from_numpy(ctx, np.zeros(16, np.float32))
    with pytest.raises(llmrs.LlmrsError):
        be.sample(d, [], 1.0, 1.0, 0.9, 1.5)


def test_model_sample_after_decode(llmrs, ctx, orc):
    from test_gpu_model import CFG_SMALL
    m = llmrs.Model(ctx, dict(CFG_SMALL, scale_dtype=0))
    m.init_synthetic(5)
    tok, logits = m.decode_step(7, 0)
    for u in (0.1, 0.5, 0.93):
        t_gpu = m.sample([7, 7, 9], 1.2, 0.8, 0.9, u)
        t_orc, margin = orc.sample(logits, [7, 7, 9], 1.2, 0.8, 0.9, u)
        assert t_gpu == t_orc or margin < 1e-6
