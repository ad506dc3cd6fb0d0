"""The autoregressive loop on the device (ming_cuda_sample_latents) and its
continuous-batching scheduler (ming_cuda_loop_*), against the oracle chaining
the flow head, the aggregator and the LM as sampleLatents does
(src/ming_model.zig:1388-1480).

Each request returns its latents and, like the reference's Trace
(src/ming_model.zig:1376-1385), the z and p(stop) of every step. The oracle
replays the chain teacher-forced on that trace: step k's latent from the
flow head on z_k, the previous latent as history and step k's noise (whole
10-step samples: max-abs 0.2, cosine > 0.999, the flow-head sample bound);
z_{k+1} and p(stop) from one oracle LM step on the aggregate of latent k
(gated like the other multi-layer LM outputs: within_reference, the 2e-2 /
0.999 tolerance widened to the reference's own FUSED-vs-GRAPH spread; p within
1e-2); and the emitted count from
the stop rule (p > 0.5 and step > 3) and the budget min(max_steps,
max_len - L) applied to the trace.

Small heads keep the oracle fast: a 2-layer 4-bit LM, 2 flow-head and 2
aggregator blocks at hidden 512. The stop head's bias sets the behaviour:
-4 never stops (runs to the budget), +4 stops at step 4.
"""
import numpy as np
import pytest

import ming_b200 as M
import oracle as O
from ming_b200 import synth

from conftest import close, within_reference

pytestmark = pytest.mark.gpu

QS = (0.002, 0.005)
DH, DB, DFF = 512, 2, 1024


def _lm(stop_bias):
    W = synth.lm_weights(seed=31, bits=4, layers=2, qscale=QS)
    W["stop_head.bias"] = synth.f32_to_bf16(np.array([0.0, stop_bias], np.float32))
    return W


def token_model(stop_bias, max_batch=8):
    Wl = _lm(stop_bias)
    Wf = synth.flow_weights(seed=32, blocks=DB, hidden=DH, ff=DFF)
    Wa = synth.agg_weights(seed=33, blocks=DB, hidden=DH, ff=DFF)
    cfg = M.default_cfg(layers=2, weight_bits=4, dit_mode=M.DIT_TOKEN, dit_hidden=DH, dit_blocks=DB, dit_heads=DH // 64,
                        dit_ff=DFF, agg_blocks=DB, dit_max_batch=max_batch, max_ctx=512, max_pages=1024,
                        max_batch=max_batch, max_seqs=16)
    ctx = M.Context(cfg, weights={**Wl, **Wf, **Wa})
    return ctx, O.Lm(Wl), O.Flow(Wf, blocks=DB, H=DH, ff=DFF), O.Agg(Wa, blocks=DB, H=DH, ff=DFF)


def noise(seed, k, width):
    """The library's seeded noise of step k: 11 rows (start noise, 10 SDE draws)."""
    return synth.normal_bf16(seed, f"loop.noise.{k}", (11, width))


def check_chain(ctx, lm, sample, embeds, hist0, seed, lat, zt, st, params, token=True):
    """Teacher-forced replay of one request's trace (see the module doc)."""
    L, n = embeds.shape[0], lat.shape[0]
    budget = min(params.max_steps, params.max_len - L)
    cache, cg = lm.new_cache(L + n + 4), lm.new_cache(L + n + 4)
    ro, rs = lm.forward(cache, embeds)
    rg, _ = lm.forward(cg, embeds, O.MODE_GRAPH)
    d, c, ok = within_reference(zt[0:1], ro[-1:], rg[-1:])
    assert ok, ("prefill z", d, c)
    assert abs(st[0] - rs[-1]) < 1e-2
    hist = hist0
    for k in range(n):
        ref = sample(zt[k], hist, noise(seed, k, lat.shape[1])[0])
        d, c, ok = close(lat[k:k + 1], ref.reshape(1, -1), tol=0.2)
        assert ok, ("latent", k, d, c)
        if k + 1 < n:
            x = ctx.aggregate(lat[k:k + 1] if token else lat[k:k + 1].reshape(1, -1, 64))
            ro, rs = lm.forward(cache, x)
            rg, _ = lm.forward(cg, x, O.MODE_GRAPH)
            d, c, ok = within_reference(zt[k + 1:k + 2], ro, rg)
            assert ok, ("z", k + 1, d, c)
            assert abs(st[k + 1] - rs[0]) < 1e-2, (k + 1, st[k + 1], rs[0])
        hist = lat[k]
    stop_at = next((k + 1 for k in range(n) if st[k] > 0.5 and k > 3), None)
    assert n == (stop_at if stop_at is not None and stop_at <= budget else budget), (n, stop_at, budget)


@pytest.fixture(scope="module")
def never_stops(cuda_ok):
    m = token_model(-4.0)
    yield m
    m[0].close()


def test_sample_latents_matches_oracle_chain(never_stops):
    ctx, lm, flow, agg = never_stops
    p = M.sample_params(max_steps=16, cfg=2.0)
    emb = synth.normal_bf16(40, "loop.prompt", (24, 896))
    pl = synth.normal_bf16(40, "loop.prompt_latent", (64,))
    lat, zt, st = ctx.sample_latents(emb, pl, p, seed=7, trace=True)
    assert lat.shape == (16, 64) and (st < 0.5).all()
    check_chain(ctx, lm, lambda z, h, nz: flow.sample(z, h, nz, None, 2.0, 0.0), emb, pl, 7, lat, zt, st, p)


def test_budget_is_max_len_minus_prompt(never_stops):
    ctx, lm, flow, agg = never_stops
    p = M.sample_params(max_steps=100, max_len=31)
    emb = synth.normal_bf16(41, "loop.prompt.b", (24, 896))
    lat, zt, st = ctx.sample_latents(emb, None, p, seed=8, trace=True)
    assert lat.shape[0] == 7  # min(100, 31 - 24)
    check_chain(ctx, lm, lambda z, h, nz: flow.sample(z, h, nz, None, 2.0, 0.0), emb, np.zeros(64, np.uint16), 8, lat,
                zt, st, p)
    with pytest.raises(M.MingError, match="too long"):
        ctx.sample_latents(synth.normal_bf16(41, "loop.long", (31, 896)), None, p, seed=8)


def test_seeded_noise_equals_its_replay_bank_and_sde(never_stops):
    """The device's seeded stream is the harness generator bit for bit: the
    same request with that noise passed as a replay bank gives the same
    latents. With temperature > 0 the SDE rows enter too (shift =
    sigma * sqrt(temperature))."""
    ctx, lm, flow, agg = never_stops
    emb = synth.normal_bf16(42, "loop.prompt.c", (12, 896))
    for temp in (0.0, 0.5):
        p = M.sample_params(max_steps=6, temperature=temp)
        a, za, sa = ctx.sample_latents(emb, None, p, seed=9, trace=True)
        bank = np.stack([noise(9, k, 64) for k in range(6)])
        b, _, _ = ctx.sample_latents(emb, None, p, bank=bank)
        assert np.array_equal(a, b), temp
        if temp:
            shift = 0.25 * np.sqrt(temp)
            hist = np.zeros(64, np.uint16)
            for k in range(6):
                nk = noise(9, k, 64)
                ref = flow.sample(za[k], hist, nk[0], nk[1:].copy(), 2.0, shift)
                d, c, ok = close(a[k:k + 1], ref.reshape(1, -1), tol=0.2)
                assert ok, ("sde latent", k, d, c)
                hist = a[k]


def test_stop_rule_ends_after_step_four(cuda_ok):
    ctx, lm, flow, agg = token_model(4.0)
    p = M.sample_params(max_steps=16)
    emb = synth.normal_bf16(43, "loop.prompt.d", (10, 896))
    lat, zt, st = ctx.sample_latents(emb, None, p, seed=10, trace=True)
    assert lat.shape[0] == 5 and (st > 0.5).all()  # emitted steps 0..4, stopped at step 4 (> 3)
    check_chain(ctx, lm, lambda z, h, nz: flow.sample(z, h, nz, None, 2.0, 0.0), emb, np.zeros(64, np.uint16), 10, lat,
                zt, st, p)
    ctx.close()


def test_loop_continuous_batching(never_stops):
    """Three rows, five requests: two wait in the queue and take the rows the
    first finishers free (budgets 12, 12, 8, 12, 12). Every request is
    replayed against the oracle chain from its own trace."""
    ctx, lm, flow, agg = never_stops
    p = M.sample_params(max_steps=12, max_len=64)
    lp = M.Loop(ctx, 3, p)
    lens = [20, 30, 56, 25, 40]
    embs = [synth.normal_bf16(44, f"loop.cb.{i}", (L, 896)) for i, L in enumerate(lens)]
    ids = [lp.submit(e, None, seed=100 + i, trace=True) for i, e in enumerate(embs)]
    active, queued = lp.step()
    assert queued == 2
    steps = 1
    res = {}
    while len(res) < len(ids):
        for i in ids:
            if i not in res:
                r = lp.result(i, trace=True)
                if r is not None:
                    res[i] = r
        if len(res) < len(ids):
            active, queued = lp.step()
            steps += 1
        assert steps < 100
    # the queued requests start as rows free up: well under running all five in turn
    assert steps <= 40
    lp.close()
    for i, L in zip(ids, lens):
        lat, zt, st = res[i]
        assert lat.shape[0] == min(12, 64 - L)
        check_chain(ctx, lm, lambda z, h, nz: flow.sample(z, h, nz, None, 2.0, 0.0), embs[ids.index(i)],
                    np.zeros(64, np.uint16), 100 + ids.index(i), lat, zt, st, p)


def test_loop_adaln_head(cuda_ok):
    """Config 5's loop shape (small): the adaLN head samples a 4-frame patch
    per step without history, the latent projection feeds the LM."""
    Wl = _lm(-4.0)
    Wd = synth.ada_weights(seed=34, blocks=DB, hidden=DH, ff=DFF)
    Wp = synth.latent_proj_weights(seed=35)
    cfg = M.default_cfg(layers=2, weight_bits=4, dit_mode=M.DIT_ADALN, dit_hidden=DH, dit_blocks=DB, dit_heads=DH // 64,
                        dit_ff=DFF, dit_frames=4, agg_blocks=0, dit_max_batch=4, max_ctx=512, max_pages=512, max_batch=4,
                        max_seqs=8)
    ctx = M.Context(cfg, weights={**Wl, **Wd, **Wp})
    lm, ada = O.Lm(Wl), O.Ada(Wd, blocks=DB, H=DH, ff=DFF, latent=64, frames=4)
    p = M.sample_params(max_steps=6)
    lp = M.Loop(ctx, 2, p)
    embs = [synth.normal_bf16(45, f"loop.ada.{i}", (16 + 8 * i, 896)) for i in range(2)]
    ids = [lp.submit(e, None, seed=200 + i, trace=True) for i, e in enumerate(embs)]
    res = {}
    for _ in range(20):
        lp.step()
        for i in ids:
            if i not in res:
                r = lp.result(i, trace=True)
                if r is not None:
                    res[i] = r
        if len(res) == 2:
            break
    lp.close()
    for j, i in enumerate(ids):
        lat, zt, st = res[i]
        assert lat.shape == (6, 256)
        check_chain(ctx, lm, lambda z, h, nz: ada.sample(z.reshape(1, -1), nz.reshape(1, 4, 64)), embs[j], None, 200 + j,
                    lat, zt, st, p, token=False)
    ctx.close()
