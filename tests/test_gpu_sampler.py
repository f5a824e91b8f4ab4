"""The device sampler (lt_sample_step) against the oracle's restatement of
src/model/sample.zig with the same DefaultPrng stream.

Bars: temperature 0 returns the first maximum and leaves the stream alone;
prompt positions leave the stream alone; every sampled step advances the
four generator words exactly as the oracle does (bit-exact); the token equals
the oracle's.  The reference accumulates the softmax denominator and the
running sums sequentially; the kernel reduces them across a thread block, so
a draw that lands within f32 rounding of a bucket edge (or a top-p cut within
rounding of top_p) may fall on the neighbour.  A differing token is accepted
only when that is shown: the float64 distribution has an edge within 1e-5 of
the draw.
"""
from __future__ import annotations

import importlib

import numpy as np
import pytest

from test_gpu_parity import dev, host

pytestmark = pytest.mark.gpu

EDGE = 1e-5


def _filtered(logits, temp, k, tp):
    """float64 restatement of sample.zig's filtering: (draw order, probs in
    that order, the prefix sums the top-p cut compares) — fast path when
    0 < k <= 256 and k < n."""
    x = logits.astype(np.float64) * (1.0 / temp if temp != 1.0 else 1.0)
    p = np.exp(x - x.max())
    p /= p.sum()
    n = p.size
    if 0 < k < n and k <= 256:
        order = np.lexsort((np.arange(n), -x))[:k]
        q = p[order]
        cuts = np.cumsum(q)
        if tp < 1.0:
            kept = int(np.argmax(cuts >= tp)) + 1 if (cuts >= tp).any() else k
            order, q = order[:kept], q[:kept]
        return order, q / q.sum(), cuts
    if 0 < k < n:
        thr = np.sort(p)[::-1][k - 1]
        p = np.where(p < thr, 0.0, p)
    cuts = np.cumsum(p[np.lexsort((np.arange(n), -p))])
    if tp < 1.0:
        srt = np.lexsort((np.arange(n), -p))
        c = np.cumsum(p[srt])
        cut = int(np.argmax(c >= tp)) + 1 if (c >= tp).any() else n
        keep = np.zeros(n, bool)
        keep[srt[:cut]] = True
        p = np.where(keep, p, 0.0)
    return np.arange(n), p / p.sum(), cuts


def _near_edge(logits, temp, k, tp, u) -> bool:
    _, q, cuts = _filtered(logits, temp, k, tp)
    c = np.cumsum(q)
    return bool(np.min(np.abs(c - u)) < EDGE or (tp < 1.0 and np.min(np.abs(cuts - tp)) < EDGE))


class _Stream:
    """A device token stream + {pos, n_prompt} word + generator words."""

    def __init__(self, pkg, seed, n_prompt=1, length=4096):
        import torch
        self.toks = torch.zeros(length, dtype=torch.int32, device="cuda")
        self.state = dev(np.array([0, n_prompt], np.int32))
        w = np.array(pkg.rng_seed(seed), np.uint64).view(np.int64)
        self.rng = dev(w)

    def words(self):
        return host(self.rng).view(np.uint64).tolist()


def _run(ctx, pkg, oracle, n, temp, k, tp, seed, draws, scale=3.0, ties=False):
    rng = np.random.default_rng(seed)
    st = _Stream(pkg, seed)
    ref = oracle.Rng(seed)
    params = pkg.SampleParams(temp, k, tp)
    near = 0
    for d in range(draws):
        lg = rng.normal(0.0, scale, n).astype(np.float32)
        if ties:
            lg = np.round(lg * 2) / 2
        lgd = dev(lg)
        ctx.sample_step(lgd, n, params, st.rng, st.toks, st.state[0:1], st.state[1:2])
        before = ref.copy()
        want = oracle.sample(lg, temp, k, tp, ref)
        got = int(host(st.toks)[d + 1])
        assert st.words() == ref.words(), d
        if got != want:
            u = before.copy().float()
            assert _near_edge(lg, temp, k, tp, u), (d, got, want, u)
            near += 1
    assert host(st.state)[0] == draws
    assert near <= max(1, draws // 50)


@pytest.mark.parametrize("n,temp,k,tp", [
    (1000, 0.8, 40, 0.9),       # the reference's fast path with nucleus
    (151936, 0.8, 40, 0.9),     # Qwen3 vocabulary
    (151936, 1.0, 256, 1.0),    # largest fast k, no nucleus
    (262144, 0.7, 1, 1.0),      # k = 1
    (5000, 1.3, 64, 0.0),       # top_p 0: the top candidate only
])
def test_fast_path_vs_oracle(ctx, pkg, oracle, n, temp, k, tp):
    _run(ctx, pkg, oracle, n, temp, k, tp, seed=n + k, draws=48)


@pytest.mark.parametrize("n,temp,k,tp", [
    (1000, 1.0, 0, 1.0),        # plain multinomial
    (151936, 0.8, 0, 0.9),      # nucleus over the whole vocabulary
    (151936, 0.8, 1000, 1.0),   # k above the fast limit: applyTopK
    (20000, 0.9, 300, 0.5),     # applyTopK then applyTopP
    (3000, 1.0, 0, 0.0),        # top_p 0 on the full path
])
def test_full_path_vs_oracle(ctx, pkg, oracle, n, temp, k, tp):
    _run(ctx, pkg, oracle, n, temp, k, tp, seed=7 * n + k, draws=32)


@pytest.mark.parametrize("k,tp", [(40, 0.9), (0, 0.8), (500, 1.0)])
def test_ties_vs_oracle(ctx, pkg, oracle, k, tp):
    """Logits on a half-integer grid: many exact ties at the top-k threshold
    and the top-p cut, which resolve in index order."""
    _run(ctx, pkg, oracle, 4000, 1.0, k, tp, seed=11 + k, draws=32, scale=1.5, ties=True)


def test_greedy_and_prompt_positions(ctx, pkg, oracle):
    """Temperature 0 is greedy (first maximum) and does not draw; prompt
    positions only advance pos."""
    st = _Stream(pkg, 5, n_prompt=3)
    w0 = st.words()
    lg = np.zeros(1000, np.float32)
    lg[[17, 600]] = 2.0
    for _ in range(2):  # prompt positions 0 and 1
        ctx.sample_step(dev(lg), 1000, pkg.SampleParams(0.8, 40, 0.9), st.rng, st.toks, st.state[0:1],
                        st.state[1:2])
    assert st.words() == w0 and host(st.state).tolist() == [2, 3]
    ctx.sample_step(dev(lg), 1000, pkg.SampleParams(0.0, 40, 0.9), st.rng, st.toks, st.state[0:1], st.state[1:2])
    assert st.words() == w0 and int(host(st.toks)[3]) == 17
    ref = oracle.Rng(5)
    ctx.sample_step(dev(lg), 1000, pkg.SampleParams(0.8, 40, 0.9), st.rng, st.toks, st.state[0:1], st.state[1:2])
    assert int(host(st.toks)[4]) == oracle.sample(lg, 0.8, 40, 0.9, ref)
    assert st.words() == ref.words() and host(st.state).tolist() == [4, 3]


def test_decoder_sampling_vs_oracle(ctx, pkg, oracle):
    """A sampled generation through the host decode loop: each step's token
    is the oracle sampler on that step's logits with the same stream, and the
    captured graph, re-seeded, replays the same tokens."""
    synth = importlib.import_module("llmtoy-zig_b200.synth")
    decoder = importlib.import_module("llmtoy-zig_b200.decoder")
    rng = np.random.default_rng(5)
    m = synth.DecoderModel(rng, 2, 256, 4, 2, 64, 500, n_experts=8, k=2, d_expert=256, lm_type=14,
                           qk_norm=True, rope_neox=True, norm_topk=True, norms_random=True)
    spec = decoder.upload_decoder(ctx, m, kv_cap=64)
    dec = decoder.Decoder(ctx, spec)
    prompt, n_gen, seed = [3, 1, 4], 12, 1234
    dec.set_sampling(0.8, 40, 0.9, seed)
    ref = oracle.Rng(seed)
    dec.start(prompt)
    toks = list(prompt)
    for i in range(len(prompt) + n_gen - 1):
        dec.step()
        lg = ctx.copy_to_host(dec.logits_ptr(), m.vocab * 4)
        if i + 1 >= len(prompt):
            toks.append(oracle.sample(lg, 0.8, 40, 0.9, ref))
    assert dec.tokens(len(toks)) == toks
    dec.set_sampling(0.8, 40, 0.9, seed)
    assert dec.generate(prompt, n_gen) == toks[len(prompt):]
    dec.set_sampling(0.8, 40, 0.9, seed)
    assert dec.generate(prompt, n_gen) == toks[len(prompt):]
    dec.set_sampling(0.0, 0, 1.0, seed)  # back to greedy: the oracle's greedy stream
    assert dec.generate(prompt, 6) == oracle.OracleDecoder(m, 64).generate(prompt, 6)[0]
    dec.close()
