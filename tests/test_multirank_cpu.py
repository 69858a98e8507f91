"""Vocabulary-split lm_head exchange on CPU ranks (gloo, world size 2 and 3).

Each rank owns the contiguous lm_head row range :func:`lm_head.vocab_shard`
gives it, computes its shard's per-row (max, argmax) with the oracle, packs
them into the kernels' 64-bit keys (:func:`lm_head.make_keys`) and exchanges
them with :func:`lm_head.gather_keys` -- the same call the GPU path makes over
NCCL.  The reduced keys must give the oracle's argmax over the full
vocabulary (``engine/sampling.py:47-55``: first index wins on ties, also when
the tied ids live on different ranks) and the oracle's acceptance
(``engine/acceptance.py:9-16``).
"""

from __future__ import annotations

import os
import socket

import numpy as np
import pytest

ROWS, DIM, VOCAB, BLOCK = 32, 64, 1001, 16


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _problem():
    """Same inputs on every rank.  Rows 0-3 have exactly tied maxima across the
    shard boundary of a 2-way split (ids 100 and 700) and 3-way split (ids 100,
    400, 900)."""
    from oracle import bf16, lmhead

    rng = np.random.default_rng(7)
    h = rng.standard_normal((ROWS, DIM)).astype(np.float32)
    w = (rng.standard_normal((VOCAB, DIM)) * 0.05).astype(np.float32)
    for vid in (100, 400, 700, 900):
        w[vid] = 0.5 * np.sign(h[0])                                  # aligned with row 0
    for r in range(1, 4):
        h[r] = h[0]
    logits = lmhead.logits_bf16(bf16.from_f32(h), bf16.from_f32(w))   # bf16 bits in
    post_full = lmhead.greedy_tokens(logits)
    ids = lmhead.synth_verify_ids(rng, post_full.reshape(-1, BLOCK), VOCAB)
    return h, w, logits, ids


def _rank_main(rank: int, world: int, port: int, q):
    import torch
    import torch.distributed as dist

    import __graft_entry__

    try:
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
        dist.init_process_group("gloo", rank=rank, world_size=world)
        pkg = __graft_entry__.load_package()
        lm = pkg.lm_head
        from oracle import lmhead

        _, _, logits, _ = _problem()
        v0, vlen = lm.vocab_shard(VOCAB, rank, world)
        if vlen:
            vals, idx = lmhead.shard_partials(logits[:, v0:v0 + vlen], v0)
        else:  # an empty shard contributes the smallest key
            vals = np.full(ROWS, -np.inf, np.float32)
            idx = np.full(ROWS, 0xFFFFFFFF, np.int64)
        keys = lm.make_keys(torch.from_numpy(vals), torch.from_numpy(idx))
        gathered = lm.gather_keys(keys, None)
        best_v, best_i = lm.decode_keys(lm.reduce_keys(gathered))
        q.put((rank, best_i.numpy().copy(), best_v.numpy().copy(), gathered.shape))
        dist.destroy_process_group()
    except BaseException as e:  # report, never hang the parent
        q.put((rank, repr(e), None, None))


def _run(world: int):
    import torch.multiprocessing as mp

    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    out = {}
    try:
        for _ in range(world):
            rank, ids, vals, shape = q.get(timeout=180)
            out[rank] = (ids, vals, shape)
    finally:
        for p in procs:
            p.join(timeout=30)
            if p.is_alive():
                p.kill()
    return out


@pytest.mark.parametrize("world", [2, 3])
def test_vocab_split_key_exchange_matches_full_argmax(world):
    from oracle import lmhead

    _, _, logits, ids = _problem()
    out = _run(world)
    full = lmhead.greedy_tokens(logits)
    assert full[0] == 100, "tie fixture: the lowest tied id must win"
    for rank in range(world):
        got, vals, shape = out[rank]
        assert not isinstance(got, str), got
        assert tuple(shape) == (world, ROWS)
        np.testing.assert_array_equal(got.astype(np.int64), full)
        np.testing.assert_array_equal(vals, logits[np.arange(ROWS), full])
    # acceptance from the exchanged argmax equals the oracle's on the full logits
    post, acc, nxt = lmhead.verify_accept(logits.reshape(-1, BLOCK, VOCAB), ids)
    got = out[0][0].reshape(-1, BLOCK)
    np.testing.assert_array_equal(got, post)
    for b in range(ids.shape[0]):
        a = lmhead.match_acceptance_length(ids[b, 1:], got[b, :-1])
        assert a == acc[b] and got[b, a] == nxt[b]


def test_vocab_shard_covers_vocabulary_once():
    import __graft_entry__

    lm = __graft_entry__.load_package().lm_head
    for vocab in (1, 7, 1001, 248320):
        for world in (1, 2, 3, 8):
            seen = np.zeros(vocab, np.int32)
            for r in range(world):
                b, n = lm.vocab_shard(vocab, r, world)
                assert n >= 0
                seen[b:b + n] += 1
            assert (seen == 1).all()
    with pytest.raises(ValueError):
        lm.vocab_shard(10, 2, 2)


def test_key_packing_orders_like_argmax():
    """make_keys / reduce_keys / decode_keys on CPU: unsigned key order is
    (value, -id) order, including infinities and subnormals; -0 and +0 tie."""
    import torch

    import __graft_entry__

    lm = __graft_entry__.load_package().lm_head
    vals = torch.tensor([1.5, -2.0, 0.0, -0.0, float("inf"), -float("inf"), 3e-39, -3e-39, 1.5])
    ids = torch.tensor([5, 1, 2, 3, 9, 4, 6, 7, 0], dtype=torch.int32)
    keys = lm.make_keys(vals, ids)
    v, i = lm.decode_keys(keys)
    assert torch.equal(v.view(torch.int32), (vals + 0.0).view(torch.int32))
    assert torch.equal(i, ids)
    # pairwise: reduce_keys picks the larger value, lower id on ties
    for a in range(len(vals)):
        for b in range(len(vals)):
            best = lm.reduce_keys(torch.stack([keys[a], keys[b]]))
            bv, bi = lm.decode_keys(best)
            va, vb = float(vals[a]), float(vals[b])
            if va > vb or (va == vb and int(ids[a]) < int(ids[b])):
                want = a
            elif vb > va or (va == vb and int(ids[b]) < int(ids[a])):
                want = b
            else:
                want = a
            assert int(bi) == int(ids[want]), (a, b)


def _step_rank_main(rank: int, world: int, port: int, q):
    """One rank of the benchmark step's multi-rank host path on gloo: the
    library is a recorder (no kernel runs), the two CUDA graphs are the
    step's parts called directly (the second holds the all-gathers, which are
    real)."""
    import contextlib
    import types

    import torch
    import torch.distributed as dist

    import __graft_entry__

    try:
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
        dist.init_process_group("gloo", rank=rank, world_size=world)
        pkg = __graft_entry__.load_package()
        from dflash_mlx_b200 import _lib, kernels, lm_head, verify_qmm, verify_step

        calls = []

        class Recorder:
            def __getattr__(self, name):
                def launch(*args):
                    calls.append(name)
                    return 0
                return launch

        _lib.load = lambda path=None: Recorder()
        for mod in (verify_qmm, lm_head, kernels, pkg.moe):
            mod.require_cuda = lambda t, name: None
            mod.stream_ptr = lambda dev: 0
            if hasattr(mod, "workspace"):
                mod.workspace = lambda dev, n: torch.zeros(16, dtype=torch.uint8)
        verify_qmm.workspace_bytes = lambda m, k, n: 16
        lm_head.workspace_bytes = lambda r, d, v: 16
        torch.cuda.Stream = lambda dev=None: None
        torch.cuda.device = lambda dev: contextlib.nullcontext()
        torch.cuda.stream = lambda s: contextlib.nullcontext()

        shape = verify_step.StackShape(hidden=256, layers=1, q_out=256, kv_out=128, inter=512, vocab=1000,
                                       gdn_layers=2, gdn_heads=2, gdn_dk=32, gdn_dv=32)
        step = verify_step.VerifyStep("cpu", requests=2, shape=shape, rank=rank, world=world, group=None,
                                      weight_layout="pairs", fuse_silu=True)
        rows = step.requests * shape.block
        step.x_all = torch.empty((world * rows, shape.hidden), dtype=torch.bfloat16)
        step.ids_all = torch.empty((world * step.requests, shape.block), dtype=torch.int32)
        step.keys_all = torch.empty((world, world * rows), dtype=torch.int64)
        step.x.fill_(rank + 1)
        step.verify_ids.fill_(10 * (rank + 1))
        parts = (step._qmm_stack, step._exchange)
        step.graphs = [types.SimpleNamespace(replay=f) for f in parts]
        calls.clear()
        step.run_step()
        q.put((rank, list(calls), step.x_all[:, 0].float().tolist(), step.ids_all[:, 0].tolist(),
               tuple(step.keys_all.shape)))
        dist.destroy_process_group()
    except BaseException as e:  # report, never hang the parent
        q.put((rank, repr(e), None, None, None))


def test_verify_step_multirank_host_path():
    """Two gloo ranks run the step's N > 1 branch: every rank issues the same
    launches in the same order, the hidden rows and verify ids of both ranks
    arrive in rank order, and the key exchange has one row of keys per rank."""
    import torch.multiprocessing as mp

    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_step_rank_main, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    out = {}
    try:
        for _ in range(world):
            rank, calls, x0, ids0, kshape = q.get(timeout=180)
            out[rank] = (calls, x0, ids0, kshape)
    finally:
        for p in procs:
            p.join(timeout=30)
            if p.is_alive():
                p.kill()
    for rank in range(world):
        calls, x0, ids0, kshape = out[rank]
        assert not isinstance(calls, str), calls
        assert calls == out[0][0]
        assert calls[-3:] == ["dfl_lmhead_argmax", "dfl_lmhead_accept", "dfl_gdn_tape_replay"]
        assert x0 == [1.0] * 32 + [2.0] * 32
        assert ids0 == [10, 10, 20, 20]
        assert kshape == (world, world * 32)
