"""The checking logic of ``__graft_entry__.smoke()``'s acceptance and rollback
parts, run on CPU with the package replaced by oracle-backed stand-ins (the
real package refuses CPU tensors): correct results pass, a planted wrong
acceptance length or state element is caught."""

from __future__ import annotations

import types

import numpy as np
import pytest
import torch

import __graft_entry__ as ge
from oracle import gdn as ogdn
from oracle import lmhead as olm


def _bits(t):
    return t.contiguous().view(torch.int16).numpy().view(np.uint16)


def _fake_pkg(bad_accept=False, bad_state=False):
    def lm_head_verify(h, w, ids):
        logits = olm.logits_bf16(_bits(h), _bits(w))
        ids = ids.numpy()
        b, t = ids.shape
        post = np.argmax(logits, axis=-1).reshape(b, t).astype(np.int32)
        acc = np.array([olm.match_acceptance_length(ids[i, 1:], post[i, :-1]) for i in range(b)], np.int32)
        nxt = post[np.arange(b), acc]
        if bad_accept:
            acc = acc.copy()
            acc[0] = (acc[0] + 1) % t
        return torch.from_numpy(post), torch.from_numpy(acc), torch.from_numpy(nxt), None

    def tape_replay_(state, tape, k, g, steps):
        out = ogdn.tape_replay_accepted(tape.numpy(), k.float().numpy(), g.numpy(), state.numpy(),
                                        steps.numpy())
        if bad_state:
            out = out.copy()
            out.reshape(-1)[7] += 1e-3
        state.copy_(torch.from_numpy(out))
        return state

    return types.SimpleNamespace(lm_head_verify=lm_head_verify,
                                 kernels=types.SimpleNamespace(tape_replay_=tape_replay_))


def test_smoke_checks_pass_on_oracle_results():
    dev = torch.device("cpu")
    assert ge._smoke_accept(_fake_pkg(), dev, np.random.default_rng(0)).startswith("accept")
    assert ge._smoke_rollback(_fake_pkg(), dev, np.random.default_rng(1)) == "rollback bit-exact"


def test_smoke_checks_catch_planted_mistakes():
    dev = torch.device("cpu")
    with pytest.raises(AssertionError):
        ge._smoke_accept(_fake_pkg(bad_accept=True), dev, np.random.default_rng(0))
    with pytest.raises(AssertionError):
        ge._smoke_rollback(_fake_pkg(bad_state=True), dev, np.random.default_rng(1))
