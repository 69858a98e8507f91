"""GPU parity of the fused lm_head argmax + greedy acceptance.

Oracle: ``oracle/lmhead.py`` (bf16 logits, argmax with the -1e9 suppress
floor, ``match_acceptance_length`` composed as in the reference's verify
tail).  Argmax ids are checked bit-exact wherever the top-2 margin of the
oracle's bf16 logits exceeds the accumulation-order tolerance (two bf16 ulps
of the winning logit); acceptance lengths and next tokens are checked
against the oracle scan applied to the kernel's own posterior and, where all
margins are clear, against the oracle's.  Also: the reference's golden
acceptance table on device, suppressed ids, vocabulary shards combined by
key max (the multi-GPU reduction), ragged row counts and BASELINE config 3
(V = 248320, D = 5120) at B = 1 and 16 on the full vocabulary and at B = 16
and 128 (256 / 2048 hidden rows) on one 8-way vocabulary shard, each with
P = 0.88 verify ids scored against the oracle's posterior.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from conftest import to_dev_bf16
from oracle import bf16 as obf16
from oracle import lmhead as olm

pytestmark = pytest.mark.gpu


def _inputs(seed, r, d, v, wscale=0.02):
    rng = np.random.default_rng(seed)
    h = obf16.from_f32(rng.standard_normal((r, d)).astype(np.float32))
    w = obf16.from_f32((rng.standard_normal((v, d)) * wscale).astype(np.float32))
    return rng, h, w


def _decode(keys):
    k = keys.cpu().numpy().astype(np.uint64)
    ids = (np.uint64(0xFFFFFFFF) - (k & np.uint64(0xFFFFFFFF))).astype(np.int64)
    return ids


def _clear(logits, ids_ref):
    best = logits[np.arange(logits.shape[0]), ids_ref]
    ulp = np.maximum(np.abs(best), 1e-3) * 2.0 ** -7
    return olm.top2_margin(logits) > 2 * ulp


@pytest.mark.parametrize("r,d,v", [(16, 256, 5000), (32, 512, 3000), (5, 128, 1000),
                                   (64, 256, 2048), (256, 128, 700), (300, 64, 520)])
def test_argmax_matches_oracle(pkg, dev, r, d, v):
    rng, h, w = _inputs(r * 7 + d + v, r, d, v)
    logits = olm.logits_bf16(h, w)
    ref = np.argmax(logits, axis=-1)
    keys = pkg.lm_head_argmax_keys(to_dev_bf16(h, dev), to_dev_bf16(w, dev))
    got = _decode(keys)
    clear = _clear(logits, ref)
    assert clear.any()
    assert np.array_equal(got[clear], ref[clear])
    # every row: the chosen id's logit is within two bf16 ulps of the maximum
    best = logits[np.arange(r), ref]
    tol = 2 * np.maximum(np.abs(best), 1e-3) * 2.0 ** -7
    assert np.all(logits[np.arange(r), got] >= best - tol)


def test_suppressed_ids_never_win(pkg, dev):
    r, d, v = 16, 256, 4000
    rng, h, w = _inputs(5, r, d, v)
    logits = olm.logits_bf16(h, w)
    top = np.argmax(logits, axis=-1)
    mask = np.zeros(v, dtype=bool)
    mask[top] = True                    # suppress every row's winner
    ref = olm.greedy_tokens(logits, mask)
    got = _decode(pkg.lm_head_argmax_keys(to_dev_bf16(h, dev), to_dev_bf16(w, dev),
                                          suppress_token_mask=torch.from_numpy(mask)))
    clear = _clear(np.where(mask[None, :], -1e9, logits).astype(np.float32), ref)
    assert not mask[got].any()
    assert np.array_equal(got[clear], ref[clear])


def test_vocab_shards_combine_to_global_argmax(pkg, dev):
    r, d, v = 32, 256, 6000
    rng, h, w = _inputs(11, r, d, v)
    th, tw = to_dev_bf16(h, dev), to_dev_bf16(w, dev)
    full = pkg.lm_head_argmax_keys(th, tw)
    bounds = [0, 1111, 2500, 4000, 6000]
    shards = torch.stack([pkg.lm_head_argmax_keys(th, tw[bounds[i]:bounds[i + 1]], v_begin=bounds[i])
                          for i in range(4)])
    post_full, _, _, mx_full = pkg.verify_accept(full, None)
    post_sh, _, _, mx_sh = pkg.verify_accept(shards, None)
    assert torch.equal(post_full, post_sh)
    assert torch.equal(mx_full, mx_sh)
    lm = pkg.lm_head
    assert torch.equal(lm.reduce_keys(shards), full)
    # the host-side key helpers use the kernels' exact key format
    vals, ids = lm.decode_keys(full)
    assert torch.equal(lm.make_keys(vals, ids), full)
    assert torch.equal(ids.cpu().long(), torch.from_numpy(_decode(full)))
    assert torch.equal(vals.reshape(-1, 16), mx_full)


def test_verify_accept_scan(pkg, dev):
    b, t, d, v = 8, 16, 256, 5000
    rng, h, w = _inputs(21, b * t, d, v)
    logits = olm.logits_bf16(h, w)
    post_ref = np.argmax(logits, axis=-1).reshape(b, t)
    ids = olm.synth_verify_ids(rng, post_ref, v, p_match=0.88)
    ids[0, 1:] = post_ref[0, :-1]          # fully accepted block
    ids[1, 1] = (post_ref[1, 0] + 1) % v   # first draft rejected
    post, acc, nxt, mx = pkg.lm_head_verify(to_dev_bf16(h, dev), to_dev_bf16(w, dev),
                                            torch.from_numpy(ids))
    post, acc, nxt = post.cpu().numpy(), acc.cpu().numpy(), nxt.cpu().numpy()
    for i in range(b):
        a = olm.match_acceptance_length(ids[i, 1:], post[i, :-1])
        assert acc[i] == a and nxt[i] == post[i, a]
    clear = _clear(logits, post_ref.reshape(-1)).reshape(b, t)
    rows = clear.all(axis=1)
    _, acc_ref, nxt_ref = olm.verify_accept(logits.reshape(b, t, v), ids)
    assert np.array_equal(acc[rows], acc_ref[rows])
    assert np.array_equal(nxt[rows], nxt_ref[rows])
    assert acc[0] == t - 1 and acc[1] == 0


@pytest.mark.parametrize("drafted,posterior,expected", [
    ([1, 2, 3, 4], [1, 2, 3, 4], 4),
    ([5, 5, 5], [1, 5, 5], 0),
    ([1, 2, 9, 4, 5], [1, 2, 3, 4, 5], 2),
    ([7, 7, 7, 0], [7, 7, 7, 1], 3),
    ([], [], 0),
])
def test_match_acceptance_golden_table_on_device(pkg, dev, drafted, posterior, expected):
    # tests/test_engine_acceptance.py:11-24
    d = torch.tensor(drafted, dtype=torch.int32, device=dev)
    p = torch.tensor(posterior, dtype=torch.int32, device=dev)
    assert int(pkg.match_acceptance_length(d, p).item()) == expected


@pytest.fixture(scope="module")
def config3_weight():
    """BASELINE config 3's lm_head, bf16 [248320, 5120] ~ N(0, 0.02), on the host."""
    v, d = 248320, 5120
    return (torch.randn(v, d, generator=torch.Generator().manual_seed(3)) * 0.02).to(torch.bfloat16)


def _check_config3(pkg, dev, h, wt, v_begin=0, seed=0):
    """Keys of one vocabulary shard against the oracle, then acceptance of
    P = 0.88 verify ids drawn against the oracle's posterior."""
    w = wt.view(torch.int16).numpy().view(np.uint16)
    logits = olm.logits_bf16(h, w)
    ref = np.argmax(logits, axis=-1)
    keys = pkg.lm_head_argmax_keys(to_dev_bf16(h, dev), wt.to(dev), v_begin=v_begin)
    got = _decode(keys) - v_begin
    clear = _clear(logits, ref)
    assert clear.mean() > 0.5
    assert np.array_equal(got[clear], ref[clear])
    r = h.shape[0]
    best = logits[np.arange(r), ref]
    tol = 2 * np.maximum(np.abs(best), 1e-3) * 2.0 ** -7
    assert np.all(logits[np.arange(r), got] >= best - tol)
    # greedy acceptance of the blocks (global ids: the shard starts at v_begin)
    b = r // 16
    rng = np.random.default_rng(seed)
    post_ref = ref.reshape(b, 16) + v_begin
    ids = olm.synth_verify_ids(rng, post_ref, v_begin + w.shape[0], p_match=0.88)
    post, acc, nxt, _ = pkg.verify_accept(keys, torch.from_numpy(ids).to(dev))
    post, acc, nxt = post.cpu().numpy(), acc.cpu().numpy(), nxt.cpu().numpy()
    for i in range(b):
        a = olm.match_acceptance_length(ids[i, 1:], post[i, :-1])
        assert acc[i] == a and nxt[i] == post[i, a]
    rows = clear.reshape(b, 16).all(axis=1)
    for i in np.flatnonzero(rows):
        assert acc[i] == olm.match_acceptance_length(ids[i, 1:], post_ref[i, :-1])
    from dflash_mlx_b200 import _lib
    assert _lib.device_error() == 0


def test_config3_full_vocab_b1(pkg, dev, config3_weight):
    rng = np.random.default_rng(3)
    h = obf16.from_f32(rng.standard_normal((16, 5120)).astype(np.float32))
    _check_config3(pkg, dev, h, config3_weight, seed=1)


def test_config3_full_vocab_b16(pkg, dev, config3_weight):
    # B = 16 verify blocks: 256 hidden rows in one launch (128-row groups)
    rng = np.random.default_rng(4)
    h = obf16.from_f32(rng.standard_normal((256, 5120)).astype(np.float32))
    _check_config3(pkg, dev, h, config3_weight, seed=2)


@pytest.mark.parametrize("r", [256, 2048])
def test_config3_vocab_shard_large_batches(pkg, dev, config3_weight, r):
    # B = 16 and B = 128 (R = 256 / 2048 rows, 256-row groups at B = 128) on the
    # 31,040-row vocabulary shard one of 8 GPUs holds (rank 3: ids 93,120..)
    v_begin, v_len = 3 * 31040, 31040
    rng = np.random.default_rng(5 + r)
    h = obf16.from_f32(rng.standard_normal((r, 5120)).astype(np.float32))
    _check_config3(pkg, dev, h, config3_weight[v_begin:v_begin + v_len].contiguous(),
                   v_begin=v_begin, seed=r)
