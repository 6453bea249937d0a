"""The densification oracle: PCG32 against the published pcg32-demo vector,
the reference's thread layout of generate_random_logistic, and the
bookkeeping of DefaultStrategy (append order, split, stable prune,
zeroed moments of appended rows, opacity reset)."""
import numpy as np
import pytest

from densify_cases import WIDTHS, make_case


def test_pcg32_known_answer(oracle):
    # pcg32_srandom(42, 54), the first outputs printed by pcg-c-basic's demo
    r = oracle.pcg32(42, 54)
    out = oracle.pcg32_next_uint(r, 6)
    assert [hex(x) for x in out] == ["0xa15c02b7", "0x7b47f409", "0xba1d3330", "0x83d2f293", "0xbfa4784b",
                                     "0xcbed606e"]


def test_pcg32_advance_equals_draws(oracle):
    a, b = oracle.pcg32(42, 1), oracle.pcg32(42, 1)
    oracle.pcg32_next_uint(a, 1000)
    oracle.pcg32_advance(b, 1000)
    assert (a.state, a.inc) == (b.state, b.inc)


def test_random_logistic_thread_layout(oracle):
    """Element idx is draw (idx % T) * 4 + idx // T, T = 128 * ceil(ceil(n/4)/128)
    (random/device.cuh:38-64), then the generator moves on by n."""
    n = 6 * 37
    r = oracle.pcg32(42, 1)
    vals = oracle.random_logistic(r, n)
    T = 128 * ((((n + 3) // 4) + 127) // 128)
    seq = oracle.pcg32(42, 1)
    draws = oracle.pcg32_next_uint(seq, 4 * T)  # thread i uses draws 4i .. 4i+3
    u = ((draws >> 9) | 0x3F800000).view(np.float32) - np.float32(1.0)
    idx = np.arange(n)
    ui = u[(idx % T) * 4 + idx // T]
    x = np.clip(ui, np.float32(1e-9), np.float32(1 - 1e-9))
    expect = (-np.log(np.float32(1.0) / x - np.float32(1.0))).astype(np.float32) * np.float32(0.551328895)
    np.testing.assert_allclose(vals, expect, rtol=1e-6, atol=1e-6)
    after = oracle.pcg32(42, 1)
    oracle.pcg32_advance(after, n)
    assert (r.state, r.inc) == (after.state, after.inc)


def test_densify_bookkeeping(oracle):
    n, cap = 4000, 8000
    params, (m, v), grads, dens = make_case(n)
    P, G = oracle.alloc_set(cap, params), oracle.alloc_set(cap, grads)
    M, V = oracle.alloc_set(cap, m), oracle.alloc_set(cap, v)
    d = np.zeros((cap, 4), np.float32)
    d[:n] = dens
    cfg = oracle.densify_config(max_screen_size=100.0 / 1280.0, reset_every=500)
    rng = oracle.pcg32(42, 1)
    new_n = oracle.densify_step(n, P, G, M, V, d, cfg, 600, rng)  # refine, prune_large on
    # expected decisions, recomputed here
    grad = dens[:, 1] / np.maximum(dens[:, 0], 1.0)
    grow = (grad > 2e-4 * 10.0) & (dens[:, 0] > 0)
    split = grow & (np.exp(params["scales"]).max(1) > 0.01)
    g = int(grow.sum())
    assert g > 0 and split.sum() > 0 and (grow & ~split).sum() > 0
    src = np.nonzero(grow)[0]
    # survivors among the n + g rows, in order
    sig = 1 / (1 + np.exp(-params["opacities"][:, 0].astype(np.float64)))
    split_sig = 1 - np.sqrt(1 - sig)  # opacity of both halves of a split
    act_all = np.concatenate([np.where(split, split_sig, sig), np.where(split[src], split_sig[src], sig[src])])
    sc = np.exp(params["scales"])
    sc_all = np.concatenate([np.where(split[:, None], sc / 1.6, sc), np.where(split[src][:, None], sc[src] / 1.6, sc[src])])
    rot_all = np.concatenate([params["rotations"], params["rotations"][src]])
    rad = np.concatenate([dens[:, 3], np.zeros(g, np.float32)])
    alive = (act_all > 0.005) & (sc_all.max(1) < 0.1) & \
            ((rad < 100.0) | (np.arange(n + g) >= n)) & (np.abs(rot_all).sum(1) > 1.1920929e-07)
    assert new_n == int(alive.sum())
    keep = np.nonzero(alive)[0]
    # stable compaction: surviving original rows keep their data (clones:
    # untouched; their sh_rest / sh0 / rotations equal the source rows)
    for k in ("sh_rest", "sh0", "rotations"):
        full = np.concatenate([params[k], params[k][src]])
        np.testing.assert_array_equal(P[k][:new_n], full[keep])
    clone_src = np.nonzero(grow & ~split)[0]
    full_means = np.concatenate([params["means"], params["means"][src]])
    unchanged = np.concatenate([~split, ~split[src]])
    np.testing.assert_array_equal(P["means"][:new_n][unchanged[keep]], full_means[keep][unchanged[keep]])
    assert clone_src.size > 0
    # moments and gradients: the appended rows are zero, the others move along
    for S, ref in ((M, m), (V, v), (G, grads)):
        for k in WIDTHS:
            full = np.concatenate([ref[k], np.zeros_like(ref[k][src])])
            np.testing.assert_array_equal(S[k][:new_n], full[keep])
    assert not d[:new_n].any()


def test_opacity_reset_step(oracle):
    n = 1000
    params, (m, v), grads, dens = make_case(n, seed=3)
    P, M, V = oracle.alloc_set(n, params), oracle.alloc_set(n, m), oracle.alloc_set(n, v)
    d = dens.copy()
    cfg = oracle.densify_config(refine_every=300, reset_every=500)
    new_n = oracle.densify_step(n, P, None, M, V, d, cfg, 1000, oracle.pcg32(42, 1))
    assert new_n == n
    sig = 1 / (1 + np.exp(-params["opacities"][:, 0].astype(np.float64)))
    expect = np.log(np.minimum(sig, 0.01) / (1 - np.minimum(sig, 0.01)))
    np.testing.assert_allclose(P["opacities"][:, 0], expect, rtol=1e-5, atol=1e-5)
    assert not M["opacities"].any() and not V["opacities"].any()
    np.testing.assert_array_equal(M["means"], m["means"])


def test_growth_past_capacity_changes_nothing(oracle):
    n = 2000
    params, (m, v), grads, dens = make_case(n, seed=5)
    P, M, V = oracle.alloc_set(n, params), oracle.alloc_set(n, m), oracle.alloc_set(n, v)
    before = {k: a.copy() for k, a in P.items()}
    cfg = oracle.densify_config()
    assert oracle.densify_step(n, P, None, M, V, dens.copy(), cfg, 500, oracle.pcg32(42, 1)) == -1
    for k in before:
        np.testing.assert_array_equal(P[k], before[k])


@pytest.mark.parametrize("step,refines", [(499, False), (500, True), (550, False), (15000, True), (15100, False)])
def test_refine_schedule(oracle, step, refines):
    n = 500
    params, (m, v), grads, dens = make_case(n, seed=11)
    P, M, V = oracle.alloc_set(2 * n, params), oracle.alloc_set(2 * n, m), oracle.alloc_set(2 * n, v)
    d = np.zeros((2 * n, 4), np.float32)
    d[:n] = dens
    new_n = oracle.densify_step(n, P, None, M, V, d, oracle.densify_config(), step, oracle.pcg32(42, 1))
    assert (new_n != n or not d[:n].any()) if refines else (new_n == n and d[:n].any())
