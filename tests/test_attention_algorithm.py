"""The online-softmax schedule of the fused attention kernel's tensor-memory
form, restated in numpy and checked against exact softmax attention (CPU).

The kernel (``attn_fwd_kernel<true>`` in csrc/attention.cu) keeps O and the
row sum l relative to a running maximum m (log2 domain) that a warp raises
only when some row of its 32 sees a block maximum more than 2^8 above its
own m; then every row of that warp rescales O and l by 2^(m_old - m_new).
Between raises the weights 2^(s - m) stay at or below 2^8.  This file runs
that schedule block by block (64 keys, 32-row warps, causal and key-length
masks) and checks O / l and the log-sum-exp against float64 softmax, on
inputs whose scores rise across blocks, so that raises happen at different
blocks for different rows.
"""

from __future__ import annotations

import numpy as np
import pytest

BN = 64        # keys per block
WARP = 32      # rows that decide a raise together
LAZY = 8.0     # log2 headroom before the maximum is raised


def _schedule(q, k, v, scale, causal, key_len=None):
    """O / l and lse (natural log) for one [S, 64] head, as the kernel's
    softmax warps compute them (fp64 arithmetic: the schedule, not rounding,
    is under test)."""
    sq, sk = q.shape[0], k.shape[0]
    if key_len is not None:
        sk = max(1, min(sk, key_len))
    scale_log2 = scale / np.log(2.0)
    out = np.zeros((sq, v.shape[1]))
    lse = np.zeros(sq)
    raises = 0
    for r0 in range(0, sq, WARP):
        rows = np.arange(r0, min(r0 + WARP, sq))
        m = np.full(len(rows), -np.inf)
        l = np.zeros(len(rows))
        o = np.zeros((len(rows), v.shape[1]))
        nkb = -(-sk // BN)
        if causal:
            nkb = min(nkb, (min(r0 + WARP, sq) - 1) // BN + 1)
        for j in range(nkb):
            key0 = j * BN
            keys = np.arange(key0, min(key0 + BN, sk))
            s = (q[rows] @ k[keys].T) * scale_log2
            vis = np.ones_like(s, dtype=bool)
            if causal:
                vis &= keys[None, :] <= rows[:, None]
            s = np.where(vis, s, -np.inf)
            mx = s.max(axis=1)
            m_new = np.maximum(m, mx)
            if np.any(m_new > m + LAZY):
                raises += 1
                use = np.where(m_new == -np.inf, 0.0, m_new)
                alpha = np.exp2(m - use)
                o *= alpha[:, None]
                l *= alpha
                m = m_new
            use = np.where(m == -np.inf, 0.0, m)
            p = np.where(vis, np.exp2(s - use[:, None]), 0.0)
            assert p.max(initial=0.0) <= 2.0 ** LAZY * (1 + 1e-12)
            o += p @ v[keys]
            l += p.sum(axis=1)
        out[rows] = o / l[:, None]
        lse[rows] = m * np.log(2.0) + np.log(l)
    return out, lse, raises


def _exact(q, k, v, scale, causal, key_len=None):
    sk = k.shape[0] if key_len is None else max(1, min(k.shape[0], key_len))
    s = (q @ k[:sk].T) * scale
    if causal:
        s = np.where(np.arange(sk)[None, :] <= np.arange(q.shape[0])[:, None], s, -np.inf)
    mx = s.max(axis=1, keepdims=True)
    e = np.exp(s - mx)
    return (e @ v[:sk]) / e.sum(axis=1, keepdims=True), (mx[:, 0] + np.log(e.sum(axis=1)))


@pytest.mark.parametrize("causal", [False, True])
@pytest.mark.parametrize("sq,sk", [(128, 256), (200, 333), (64, 1024)])
def test_lazy_rescale_schedule_matches_softmax(causal, sq, sk):
    rng = np.random.default_rng(sq * 7 + sk + causal)
    q = rng.standard_normal((sq, 64))
    # keys whose scores climb from block to block: the running maximum has
    # to be raised several times, at different blocks for different rows
    k = rng.standard_normal((sk, 64)) * (1.0 + 3.0 * np.arange(sk)[:, None] / sk)
    v = rng.standard_normal((sk, 64))
    if causal and sq != sk:
        sq = min(sq, sk)
        q = q[:sq]
    scale = 1.0
    got, got_lse, raises = _schedule(q, k, v, scale, causal)
    want, want_lse = _exact(q, k, v, scale, causal)
    assert raises >= 2
    np.testing.assert_allclose(got, want, rtol=1e-10, atol=1e-12)
    np.testing.assert_allclose(got_lse, want_lse, rtol=1e-12, atol=1e-10)


@pytest.mark.parametrize("key_len", [1, 63, 64, 65, 300])
def test_key_length_limit(key_len):
    rng = np.random.default_rng(key_len)
    q = rng.standard_normal((1, 64))
    k = rng.standard_normal((512, 64))
    v = rng.standard_normal((512, 64))
    got, got_lse, _ = _schedule(q, k, v, 0.125, False, key_len)
    want, want_lse = _exact(q, k, v, 0.125, False, key_len)
    np.testing.assert_allclose(got, want, rtol=1e-10, atol=1e-12)
    np.testing.assert_allclose(got_lse, want_lse, rtol=1e-12, atol=1e-10)


def test_scores_that_fall_need_no_raise():
    """Scores that only fall after the first block never raise the maximum
    again: one raise (the first visible block), and the result is exact."""
    rng = np.random.default_rng(3)
    q = rng.standard_normal((32, 64))
    k = rng.standard_normal((256, 64)) * np.where(np.arange(256) < BN, 3.0, 0.05)[:, None]
    v = rng.standard_normal((256, 64))
    got, _, raises = _schedule(q, k, v, 1.0, False)
    want, _ = _exact(q, k, v, 1.0, False)
    assert raises == 1
    np.testing.assert_allclose(got, want, rtol=1e-10, atol=1e-12)
