"""Host-side logic on CPU, checked against the reference's own test data.

* ``tests/golden/reference_cases.json`` (read from the dflash-mlx test sources
  by ``tests/golden/make_golden.py``): the acceptance table, the qmm parity
  harness's shapes and random-shape rule, the verify-linear eligibility shapes;
* rollback control (``engine/target_qwen_gdn.py:1003-1066``) with the fake
  cache entries of ``tests/test_engine_rollback.py``;
* verify-linear eligibility and installation (``verify_linear.py:54-87,
  338-361``) on CPU-held modules (no kernel runs).
"""

from __future__ import annotations

import json
from pathlib import Path

import numpy as np
import pytest
import torch
from torch import nn

import __graft_entry__
from oracle import lmhead as olm

GOLDEN = json.loads((Path(__file__).resolve().parent / "golden" / "reference_cases.json").read_text())


@pytest.fixture(scope="module")
def pkg():
    return __graft_entry__.load_package()


# ------------------------------------------------------------ golden data
@pytest.mark.parametrize("case", GOLDEN["acceptance_cases"])
def test_acceptance_table_from_reference_tests(case):
    got = olm.match_acceptance_length(np.array(case["drafted"], np.uint32),
                                      np.array(case["posterior"], np.uint32))
    assert got == case["expected"]


def test_qmm_random_shapes_follow_reference_rule():
    """The GPU parity suite's random shapes are the reference harness's."""
    from test_qmm_gpu import _gen_random_shapes

    rule = GOLDEN["qmm_random_shapes"]
    rng = np.random.default_rng(rule["seed"])
    gs = GOLDEN["qmm_group_size"]
    expected = []
    for i in range(rule["n"]):
        m = rule["m_levels"][i % len(rule["m_levels"])]
        k = int(rng.integers(*rule["k_blocks_range"])) * gs
        n = int(rng.integers(*rule["n_blocks_range"])) * 8
        expected.append((f"rnd{i:02d}", m, k, n))
    assert _gen_random_shapes(rule["n"], rule["seed"]) == expected


def test_qmm_real_shapes_cover_reference_lists():
    from test_qmm_gpu import REAL_SHAPES, REAL_M4_SHAPES

    ours = {(m, k, n) for _, m, k, n in REAL_SHAPES + REAL_M4_SHAPES}
    for _, m, k, n in GOLDEN["qmm_real_mlp_shapes"] + GOLDEN["qmm_real_mlp_m4_shapes"]:
        assert (m, k, n) in ours


# ------------------------------------------------------------ rollback control
class _ArmableCache:
    def __init__(self):
        self.armed_at: list[int] = []
        self.rolled_back_to: list[int] = []
        self._tape, self._tape_k, self._tape_g, self._tape_qkv = "x", "y", "z", "q"
        self._snapshot = "s"
        self._armed = True

    def arm_rollback(self, *, prefix_len: int) -> None:
        self.armed_at.append(int(prefix_len))

    def rollback(self, accepted: int) -> None:
        self.rolled_back_to.append(int(accepted))

    def clear_transients(self) -> None:
        self._tape = self._tape_k = self._tape_g = self._tape_qkv = self._snapshot = None
        self._armed = False


class _OffsetCache:
    def __init__(self, offset: int):
        self.offset = int(offset)
        self.trim_calls: list[int] = []

    def trim(self, n: int) -> None:
        self.trim_calls.append(int(n))
        self.offset -= int(n)


class _CropCache:
    def __init__(self):
        self.crop_calls: list[int] = []

    def crop(self, target_len: int) -> None:
        self.crop_calls.append(int(target_len))


def test_arm_calls_arm_rollback_with_int_prefix(pkg):
    a, b = _ArmableCache(), _ArmableCache()
    pkg.arm_rollback([a, b, "not_armable"], prefix_len=42)
    assert a.armed_at == [42] and b.armed_at == [42]


def test_clear_rollback_state_uses_clear_transients(pkg):
    c = _ArmableCache()
    pkg.clear_rollback_state(c)
    assert c._armed is False and c._tape is None and c._tape_k is None and c._snapshot is None


def test_full_acceptance_skips_replay(pkg):
    c = _ArmableCache()
    ns = pkg.restore_after_acceptance([c], target_len=100, acceptance_length=4, drafted_tokens=4)
    assert c.rolled_back_to == [] and c._tape is None and ns == 0


def test_partial_acceptance_rolls_back_to_acceptance_length(pkg):
    c = _ArmableCache()
    ns = pkg.restore_after_acceptance([c], target_len=100, acceptance_length=2, drafted_tokens=4)
    assert c.rolled_back_to == [2] and ns >= 0


def test_offset_caches_trim_to_target(pkg):
    over, under = _OffsetCache(110), _OffsetCache(80)
    pkg.restore_after_acceptance([over, under], target_len=100, acceptance_length=0,
                                 drafted_tokens=0)
    assert over.trim_calls == [10] and under.trim_calls == []


def test_crop_fallback(pkg):
    c = _CropCache()
    pkg.restore_after_acceptance([c], target_len=64, acceptance_length=0, drafted_tokens=0)
    assert c.crop_calls == [64]


def test_cleanup_clears_transients_and_empties_lists(pkg):
    c = _ArmableCache()
    target, draft = [c], ["draft_entry"]
    pkg.cleanup_generation_caches(target, draft)
    assert target == [] and draft == [] and c._tape is None


def test_rollback_cache_without_tape_restores_snapshot(pkg):
    """Rollback with no recorded tape restores the armed snapshot (CPU tensors,
    no replay kernel involved) and clears the transients."""
    cache = pkg.RecurrentRollbackCache(2)
    cache[0] = torch.ones(2, 3)
    cache[1] = torch.zeros(2, 4)
    cache.arm_rollback(prefix_len=5)
    cache[0] = torch.full((2, 3), 7.0)
    cache.rollback(1)
    assert torch.equal(cache[0], torch.ones(2, 3))
    assert cache._tape is None and cache._snapshot is None


# ------------------------------------------------------------ verify linears
def _ql(pkg, n, k, *, bits=4, group_size=64, mode="affine"):
    w = torch.zeros((n, k * bits // 32), dtype=torch.int32)
    s = torch.ones((n, k // group_size), dtype=torch.bfloat16)
    return pkg.QuantizedLinear(w, s, s.clone(), group_size=group_size, bits=bits, mode=mode)


def test_eligibility_basic_and_large_n(pkg):
    small = GOLDEN["linear_small"]
    assert pkg.is_verify_eligible(_ql(pkg, small["out_dims"], small["in_dims"]))
    assert not pkg.is_verify_eligible(_ql(pkg, GOLDEN["linear_large_n"], small["in_dims"]))


def test_eligibility_rejects_layouts_without_a_kernel(pkg):
    assert not pkg.is_verify_eligible(_ql(pkg, 64, 512, bits=8))
    assert not pkg.is_verify_eligible(_ql(pkg, 64, 512, group_size=32))
    assert not pkg.is_verify_eligible(_ql(pkg, 64, 512, mode="mxfp4"))
    assert not pkg.is_verify_eligible(nn.Linear(8, 8))


def test_eligibility_include_filter(pkg, monkeypatch):
    ql = _ql(pkg, 64, 512)
    monkeypatch.setenv("DFLASH_VERIFY_INCLUDE", "mlp")
    assert pkg.is_verify_eligible(ql, path="model.layers.0.mlp.gate_proj")
    assert not pkg.is_verify_eligible(ql, path="model.layers.0.self_attn.q_proj")
    monkeypatch.setenv("DFLASH_VERIFY_INCLUDE", "attn_q,gdn")
    assert pkg.is_verify_eligible(ql, path="model.layers.0.self_attn.q_proj")
    assert pkg.is_verify_eligible(ql, path="model.layers.3.linear_attn.out_proj")
    assert not pkg.is_verify_eligible(ql, path="model.layers.0.self_attn.k_proj")
    monkeypatch.setenv("DFLASH_VERIFY_MAX_N", "32")
    assert not pkg.is_verify_eligible(ql, path="model.layers.0.self_attn.q_proj")


def test_install_swaps_eligible_modules_once(pkg):
    class Block(nn.Module):
        def __init__(self):
            super().__init__()
            self.gate_proj = _ql(pkg, 128, 512)
            self.down_proj = _ql(pkg, 512, 128)
            self.wide = _ql(pkg, 64, 512, bits=8)              # no kernel: stays

    model = nn.Module()
    model.mlp = Block()
    model.head = nn.Linear(4, 4)
    w_ptr = model.mlp.gate_proj.weight.data_ptr()
    n = pkg.install_verify_linears(model)
    assert n == 2
    assert isinstance(model.mlp.gate_proj, pkg.VerifyQuantizedLinear)
    assert isinstance(model.mlp.down_proj, pkg.VerifyQuantizedLinear)
    assert not isinstance(model.mlp.wide, pkg.VerifyQuantizedLinear)
    assert pkg.install_verify_linears(model) == 0
    # the wrapper shares the original (already contiguous) tensors
    assert model.mlp.gate_proj.weight.data_ptr() == w_ptr
    only_down = nn.Module()
    only_down.mlp = Block()
    assert pkg.install_verify_linears(only_down, predicate=lambda path, m: path.endswith("down_proj")) == 1


# ------------------------------------------------------------ stream-K split
@pytest.mark.parametrize("total", [1, 2, 3, 147, 148, 149, 296, 480, 640, 1360, 2720, 3392, 99999])
def test_stream_k_ranges_cover_every_unit_once(pkg, total):
    """The split the qmm launches use (host code of the library, no device):
    ranges are contiguous, non-empty, cover [0, total) exactly once, and the
    later CTAs (which start last under programmatic launch) never get more
    units than the first half."""
    import ctypes

    from dflash_mlx_b200 import _lib

    grid = min(total, 148)
    ubeg = (ctypes.c_int * (grid + 1))()
    skew = ctypes.c_int(-1)
    assert _lib.load().dfl_qmm_stream_k_ranges(total, grid, ubeg, ctypes.byref(skew)) == 0
    u = np.array(list(ubeg))
    n = np.diff(u)
    assert u[0] == 0 and u[-1] == total
    assert (n >= 1).all()
    assert 0 <= skew.value <= 255
    if skew.value > 0:
        h = grid // 2
        assert n[h:].max() <= n[:h].max()
        assert n[-1] <= n[0]


def test_stream_k_ranges_reject_bad_input(pkg):
    import ctypes

    from dflash_mlx_b200 import _lib

    ubeg = (ctypes.c_int * 8)()
    assert _lib.load().dfl_qmm_stream_k_ranges(3, 5, ubeg, None) == 2   # grid > total
    assert _lib.load().dfl_qmm_stream_k_ranges(0, 1, ubeg, None) == 2


# ------------------------------------------------------------ byte accounting
def test_stack_bytes_per_layer_match_launch_shapes(pkg):
    """The roofline's algorithmic bytes: per launch, packed nibbles N K / 2,
    bf16 scales and biases 2 x 2 N K / 64, bf16 rows in and out 2 x 16 x
    (K + N_out), with N_out = N / 2 for the fused gate|up + SiLU launch.  For
    the benchmark's decoder layer (q|k|v 8192 x 5120, o 5120 x 6144, gate|up
    34816 x 5120, down 5120 x 17408) that is 193,921,024 bytes."""
    from dflash_mlx_b200.verify_step import StackShape

    def launch_bytes(n, k, n_out):
        return n * k // 2 + 4 * n * (k // 64) + 2 * 16 * (k + n_out)

    expect = (launch_bytes(8192, 5120, 8192) + launch_bytes(5120, 6144, 5120)
              + launch_bytes(34816, 5120, 17408) + launch_bytes(5120, 17408, 5120))
    assert expect == 193_921_024
    one = StackShape(layers=1)
    assert one.qmm_bytes_per_request(silu_fused=True) == expect
    assert one.qmm_bytes_per_step(1, 2, silu_fused=True) == expect
    assert StackShape().qmm_bytes_per_step(1, 8, silu_fused=True) == 64 * expect


@pytest.mark.parametrize("requests", [1, 2, 3, 8, 9, 64])
def test_stack_bytes_count_weights_once_per_shared_launch(pkg, requests):
    """Requests whose rows share each launch read the weights once per group:
    ceil(requests / 2) times with the per-call kernel's 32-row tile, ceil(
    requests / 8) times with the plan's 128-row tile; activations are per
    request either way."""
    from dflash_mlx_b200.verify_step import StackShape

    sh = StackShape(layers=2)
    per_req = sh.qmm_bytes_per_request(silu_fused=True)
    acts = sum(2 * sh.block * (k + (n // 2 if name == "gate_up" else n))
               for name, n, k in sh.launches()) * sh.layers
    weights = per_req - acts
    assert sh.qmm_bytes_per_step(requests, 1, silu_fused=True) == requests * per_req
    for per_launch in (2, 8):
        assert (sh.qmm_bytes_per_step(requests, per_launch, silu_fused=True)
                == -(-requests // per_launch) * weights + requests * acts)


def test_device_error_clears_cached_workspaces(pkg, monkeypatch):
    """A reported device error zeroes the cached workspaces (a timed-out
    kernel may have left partial sums); no error leaves them alone.  The
    library call is faked: no device is involved."""
    from dflash_mlx_b200 import _lib, _runtime

    word = {"v": 0}

    class FakeLib:
        def dfl_get_device_error(self, ptr):
            ptr._obj.value = word["v"]
            return 0

    monkeypatch.setattr(_lib, "load", lambda path=None: FakeLib())
    bufs = {(0, 1): torch.full((64,), 7, dtype=torch.uint8), (0, 2): torch.full((32,), 9, dtype=torch.uint8)}
    monkeypatch.setattr(_runtime, "_workspaces", bufs)
    assert _lib.device_error() == 0
    assert all(int(b.sum()) > 0 for b in bufs.values())
    word["v"] = 3
    assert _lib.device_error() == 3
    assert all(int(b.sum()) == 0 for b in bufs.values())


# ------------------------------------------------------------ load-time layouts
def test_interleave_gate_up_row_order(pkg):
    """Rows [g0..g15, u0..u15, g16..g31, u16..u31, ...] along the chosen dim;
    the expert-stack form interleaves each expert on its own."""
    from dflash_mlx_b200.verify_qmm import interleave_gate_up

    gate = torch.arange(48 * 3, dtype=torch.int32).reshape(48, 3)
    up = -1 - gate
    out = interleave_gate_up(gate, up)
    assert out.shape == (96, 3)
    for blk in range(3):
        assert torch.equal(out[32 * blk:32 * blk + 16], gate[16 * blk:16 * blk + 16])
        assert torch.equal(out[32 * blk + 16:32 * blk + 32], up[16 * blk:16 * blk + 16])
    eg = torch.arange(2 * 32 * 4, dtype=torch.int32).reshape(2, 32, 4)
    eu = eg + 1000
    stacked = interleave_gate_up(eg, eu, dim=-2)
    for e in range(2):
        assert torch.equal(stacked[e], interleave_gate_up(eg[e], eu[e]))
    qe = pkg.moe.QuantWeight(eg, eg[..., :1].to(torch.bfloat16), eg[..., 1:2].to(torch.bfloat16))
    qu = pkg.moe.QuantWeight(eu, eu[..., :1].to(torch.bfloat16), eu[..., 1:2].to(torch.bfloat16))
    fused = pkg.moe.fuse_expert_gate_up(qe, qu)
    assert torch.equal(fused.q, stacked)
    assert torch.equal(fused.s, interleave_gate_up(qe.s, qu.s, dim=-2))
    with pytest.raises(ValueError):
        interleave_gate_up(gate[:40], up[:40])
    with pytest.raises(ValueError):
        interleave_gate_up(gate, up[:32])


def test_moe_helpers_refuse_bad_arguments_before_any_launch(pkg, monkeypatch):
    """gather_qmm / silu_mul / combine check dtypes, shapes and layouts on the
    host.  The CUDA-residency check is lifted so CPU tensors reach the other
    checks; every case here is refused before the library is asked to launch."""
    from dflash_mlx_b200 import moe

    monkeypatch.setattr(moe, "require_cuda", lambda t, name: None)
    bf, i32 = torch.bfloat16, torch.int32
    e, n, k = 4, 64, 128

    def stack(n_=n, k_=k, sdt=bf):
        return moe.QuantWeight(torch.zeros((e, n_, k_ // 8), dtype=i32), torch.zeros((e, n_, k_ // 64), dtype=sdt),
                               torch.zeros((e, n_, k_ // 64), dtype=sdt))

    table = torch.zeros(int(moe._lib.load().dfl_moe_route_table_ints(e)), dtype=i32)
    x = torch.zeros((16, k), dtype=bf)
    cases = {
        "x width": lambda: moe.gather_qmm(torch.zeros((16, 64), dtype=bf), stack(), table, rows_out=32,
                                          gather_by_pair=False),
        "x dtype": lambda: moe.gather_qmm(x.float(), stack(), table, rows_out=32, gather_by_pair=False),
        "scales dtype": lambda: moe.gather_qmm(x, stack(sdt=torch.float16), table, rows_out=32,
                                               gather_by_pair=False),
        "scales shape": lambda: moe.gather_qmm(
            x, moe.QuantWeight(stack().q, torch.zeros((e, n, 1), dtype=bf), torch.zeros((e, n, 1), dtype=bf)),
            table, rows_out=32, gather_by_pair=False),
        "non-contiguous q": lambda: moe.gather_qmm(
            x, moe.QuantWeight(torch.zeros((e, k // 8, n), dtype=i32).transpose(1, 2), stack().s, stack().b),
            table, rows_out=32, gather_by_pair=False),
        "short table": lambda: moe.gather_qmm(x, stack(), table[:8], rows_out=32, gather_by_pair=False),
        "pair rows": lambda: moe.gather_qmm(x, stack(), table, rows_out=32, gather_by_pair=True),
        "out shape": lambda: moe.gather_qmm(x, stack(), table, rows_out=32, gather_by_pair=False,
                                            out=torch.zeros((32, n + 1), dtype=bf)),
        "silu dtype": lambda: moe.silu_mul(torch.zeros(16, 8, dtype=torch.float16),
                                           torch.zeros(16, 8, dtype=torch.float16)),
        "silu shapes": lambda: moe.silu_mul(torch.zeros(16, 8, dtype=bf), torch.zeros(16, 9, dtype=bf)),
        "combine weights dtype": lambda: moe.combine(torch.zeros((32, 8), dtype=bf), torch.zeros((16, 2), dtype=bf),
                                                     None),
        "combine rows": lambda: moe.combine(torch.zeros((31, 8), dtype=bf), torch.zeros((16, 2)), None),
        "combine shared": lambda: moe.combine(torch.zeros((32, 8), dtype=bf), torch.zeros((16, 2)),
                                              torch.zeros((16, 9), dtype=bf)),
    }
    for name, call in cases.items():
        with pytest.raises(ValueError):
            call()
            pytest.fail(name)


@pytest.mark.parametrize("fused,shared", [(False, False), (False, True), (True, True), (True, False)])
@pytest.mark.parametrize("e,hid,inter,top_k", [(256, 2048, 512, 8), (16, 512, 256, 4), (8, 512, 128, 2)])
def test_moe_layer_valid_arguments_pass_host_checks(pkg, monkeypatch, fused, shared, e, hid, inter, top_k):
    """The argument checks accept every call a MoE layer makes (BASELINE
    config 2 and the GPU suite's smaller layers; fused and unfused gate/up,
    with and without the shared expert).  The library is replaced by a
    recorder: no kernel runs, only the launches that would be issued are
    listed."""
    from dflash_mlx_b200 import moe, verify_qmm

    real = moe._lib.load()
    calls = []

    class Recorder:
        def __getattr__(self, name):
            if name.endswith(("_workspace_bytes", "_table_ints")):
                return getattr(real, name)

            def launch(*args):
                calls.append(name)
                return 0
            return launch

    for mod in (moe, verify_qmm):
        monkeypatch.setattr(mod, "require_cuda", lambda t, name: None)
        monkeypatch.setattr(mod, "stream_ptr", lambda dev: 0)
    monkeypatch.setattr(moe._lib, "load", lambda path=None: Recorder())
    monkeypatch.setattr(moe, "workspace", lambda dev, n: torch.zeros(max(n, 1), dtype=torch.uint8))
    monkeypatch.setattr(verify_qmm, "workspace", lambda dev, n: torch.zeros(max(n, 1), dtype=torch.uint8))
    monkeypatch.setattr(verify_qmm, "workspace_bytes", lambda m, k, n: 1 << 16)
    monkeypatch.setattr(moe, "_moe_ws_bytes", lambda mp, k, n: 1 << 16)
    monkeypatch.setattr(torch.cuda, "device", lambda d: __import__("contextlib").nullcontext())

    t = 16

    def qw(n, k, lead=()):
        return moe.QuantWeight(torch.zeros((*lead, n, k // 8), dtype=torch.int32),
                               torch.zeros((*lead, n, k // 64), dtype=torch.bfloat16),
                               torch.zeros((*lead, n, k // 64), dtype=torch.bfloat16))

    experts = {"gate": qw(inter, hid, (e,)), "up": qw(inter, hid, (e,)), "down": qw(hid, inter, (e,))}
    sh = {"gate": qw(inter, hid), "up": qw(inter, hid), "down": qw(hid, inter)} if shared else None
    if fused:
        il = verify_qmm.interleave_gate_up
        experts = {"gate_up": moe.fuse_expert_gate_up(experts["gate"], experts["up"]), "down": experts["down"]}
        if sh is not None:
            g, u = sh["gate"], sh["up"]
            sh = {"gate_up": moe.QuantWeight(il(g.q, u.q).contiguous(), il(g.s, u.s).contiguous(),
                                             il(g.b, u.b).contiguous()), "down": sh["down"]}
    x = torch.zeros((t, hid), dtype=torch.bfloat16)
    y = moe.moe_layer(x, torch.zeros((t, e)), experts, sh, top_k=top_k)
    assert tuple(y.shape) == (t, hid)
    grouped = [c for c in calls if c.startswith("dfl_moe_qmm")]
    assert calls[0] == "dfl_moe_route" and calls[-1] == "dfl_moe_combine"
    assert grouped == (["dfl_moe_qmm_w4g64_silu", "dfl_moe_qmm_w4g64"] if fused else ["dfl_moe_qmm_w4g64"] * 3)


def test_qmm_wrappers_refuse_mismatched_outputs(pkg, monkeypatch):
    """A caller-provided ``out`` must be exactly what the kernel writes
    (contiguous, shape, dtype); ``repack_pairs(w, out=w)`` never writes into a
    contiguous copy.  Refused on the host, before any launch."""
    from dflash_mlx_b200 import verify_qmm

    monkeypatch.setattr(verify_qmm, "require_cuda", lambda t, name: None)
    bf = torch.bfloat16
    x = torch.zeros((16, 128), dtype=bf)
    w = torch.zeros((64, 16), dtype=torch.int32)
    s = torch.zeros((64, 2), dtype=bf)
    for bad in (torch.zeros((16, 63), dtype=bf), torch.zeros((16, 64), dtype=torch.float16),
                torch.zeros((64, 16), dtype=bf).t()):
        with pytest.raises(ValueError):
            verify_qmm.qmm_w4g64(x, w, s, s, out=bad)
    with pytest.raises(ValueError):
        verify_qmm.gate_up_silu(x, w, s, s, out=torch.zeros((16, 64), dtype=bf))
    with pytest.raises(ValueError):
        verify_qmm.repack_pairs(w, out=torch.zeros((16, 64), dtype=torch.int32).t())
    with pytest.raises(ValueError):
        verify_qmm.repack_pairs(w, out=torch.zeros((64, 16), dtype=torch.int64))


def _split_k_protocol(ubeg, ku):
    """Host model of the dense qmm's split-K hand-off (one CTA per range
    ``[ubeg[c], ubeg[c + 1])`` of (tile, K unit) pairs, ``ku`` units per
    tile): which CTA writes a partial slot for which tile, and which CTA
    reduces which slots.  Mirrors the kernel's rules: a tile's owner is the
    CTA holding its first unit; a shared tile is the last of its owner's
    range; the owner sums the slots of CTAs owner+1 .. (CTA of the tile's
    last unit)."""
    grid = len(ubeg) - 1

    def cta_of(u):
        return int(np.searchsorted(ubeg, u, side="right") - 1)

    writes, reads, finals = {}, {}, {}
    for c in range(grid):
        u0, u1 = ubeg[c], ubeg[c + 1]
        for t in range(u0 // ku, (u1 - 1) // ku + 1):
            kb0 = max(u0, t * ku) - t * ku
            kb1 = min(u1, (t + 1) * ku) - t * ku
            if kb0 == 0 and kb1 == ku:
                finals.setdefault(t, []).append(c)
            elif cta_of(t * ku) != c:
                writes.setdefault(c, []).append(t)
            else:
                assert t == (u1 - 1) // ku, "a shared tile is the last of its owner's range"
                reads[c] = (t, list(range(c + 1, cta_of(t * ku + ku - 1) + 1)))
                finals.setdefault(t, []).append(c)
    return writes, reads, finals


@pytest.mark.parametrize("n_tiles,ku", [(1, 1), (1, 12), (3, 34), (40, 12), (64, 10), (80, 10),
                                        (148, 1), (149, 1), (272, 10), (40, 34), (8, 2), (640, 4)])
def test_split_k_slots_written_once_and_reduced_once(pkg, n_tiles, ku):
    """On the library's own ranges (dfl_qmm_stream_k_ranges) for the
    benchmark's launch shapes and edge cases: every tile gets exactly one
    final store; each CTA writes at most one partial slot; every written slot
    is read by exactly one reducer, for the tile it was written for, and
    every slot a reducer reads was written."""
    import ctypes

    from dflash_mlx_b200 import _lib

    total = n_tiles * ku
    grid = min(total, 148)
    ubeg = (ctypes.c_int * (grid + 1))()
    assert _lib.load().dfl_qmm_stream_k_ranges(total, grid, ubeg, None) == 0
    writes, reads, finals = _split_k_protocol(np.array(list(ubeg)), ku)
    assert sorted(finals) == list(range(n_tiles))
    assert all(len(v) == 1 for v in finals.values())
    assert all(len(v) == 1 for v in writes.values())
    read_by = {}
    for owner, (t, srcs) in reads.items():
        for c in srcs:
            assert c not in read_by, "a slot is reduced twice"
            read_by[c] = owner
            assert writes.get(c) == [t], f"CTA {c} holds no partial of tile {t}"
    assert set(read_by) == set(writes)


@pytest.mark.parametrize("problems,tpp,ku", [(0, 8, 4), (1, 8, 4), (3, 8, 4), (37, 8, 4), (102, 8, 4),
                                             (1, 16, 1), (5, 16, 1), (102, 16, 1), (128, 4, 1),
                                             (7, 1, 34), (200, 2, 3)])
def test_grouped_split_k_even_ranges(problems, tpp, ku):
    """Grouped (MoE) launches know their unit count only on the device and
    cut it evenly over a grid sized for the largest count (CTA c starts at
    floor(c * total / grid)), so CTAs may get empty ranges.  The closed-form
    owner of a unit the kernel uses, ceil((u + 1) grid / total) - 1, is the
    last CTA whose range starts at or before u (hence a non-empty one), and
    the hand-off invariants hold with empty ranges."""
    grid = 148
    total = problems * tpp * ku
    ubeg = np.array([c * total // grid for c in range(grid + 1)])
    for u in range(total):
        closed = ((u + 1) * grid + total - 1) // total - 1
        assert closed == int(np.searchsorted(ubeg, u, side="right") - 1)
        assert ubeg[closed] <= u < ubeg[closed + 1]
    writes, reads, finals = _split_k_protocol(ubeg, ku)
    assert sorted(finals) == list(range(problems * tpp))
    assert all(len(v) == 1 for v in finals.values())
    assert all(len(v) == 1 for v in writes.values())
    read = [c for _, srcs in reads.values() for c in srcs]
    assert sorted(read) == sorted(writes)
    for owner, (t, srcs) in reads.items():
        assert all(writes[c] == [t] for c in srcs)


def test_replay_refuses_step_counts_and_masks_of_the_wrong_size(pkg, monkeypatch):
    """The replay kernel reads one step count per sequence and one mask byte
    per (sequence, step): other sizes are refused on the host."""
    from dflash_mlx_b200 import kernels

    monkeypatch.setattr(kernels, "require_cuda", lambda t, name: None)
    b, t, h, d = 3, 4, 2, 32
    tape = torch.zeros((b, t, h, d))
    k = torch.zeros((b, t, h, d), dtype=torch.bfloat16)
    g = torch.ones((b, t, h))
    state = torch.zeros((b, h, d, d))
    with pytest.raises(ValueError):
        kernels.tape_replay_(state, tape, k, g, torch.ones(1, dtype=torch.int32))
    with pytest.raises(ValueError):
        kernels.tape_replay_(state, tape, k, g, torch.ones(b + 1, dtype=torch.int32))
    with pytest.raises(ValueError):
        kernels.tape_replay_kernel(tape, k, g, state, torch.ones((b, t - 1), dtype=torch.bool))


def test_tree_conv_refuses_mismatched_bias_and_prefix(pkg, monkeypatch):
    from dflash_mlx_b200 import kernels

    seen = []
    monkeypatch.setattr(kernels, "require_cuda", lambda t, name: seen.append(name))
    qkv = torch.zeros((1, 4, 8))
    prefix = torch.zeros((1, 3, 8))
    w = torch.ones((8, 4, 1))
    path = torch.zeros((4, 4), dtype=torch.int32)
    with pytest.raises(ValueError):
        kernels.tree_depthwise_conv1d(qkv, prefix, w, torch.zeros(7), path)
    assert "prefix" in seen  # the prefix is read by the kernel: it must be on the device too
    with pytest.raises(ValueError):
        kernels.tree_depthwise_conv1d(qkv, torch.zeros((1, 2, 8)), w, None, path)


def test_lm_head_keys_refuse_bad_outputs_and_offsets(pkg, monkeypatch):
    from dflash_mlx_b200 import lm_head

    monkeypatch.setattr(lm_head, "require_cuda", lambda t, name: None)
    h = torch.zeros((16, 64), dtype=torch.bfloat16)
    w = torch.zeros((100, 64), dtype=torch.bfloat16)
    for bad in (torch.zeros(15, dtype=torch.int64), torch.zeros(16, dtype=torch.int32),
                torch.zeros((16, 2), dtype=torch.int64)[:, 0]):
        with pytest.raises(ValueError):
            lm_head.lm_head_argmax_keys(h, w, out=bad)
    with pytest.raises(ValueError):
        lm_head.lm_head_argmax_keys(h, w, v_begin=-1)
    with pytest.raises(ValueError):
        lm_head.lm_head_argmax_keys(h, w, v_begin=10, suppress_token_mask=torch.zeros(100, dtype=torch.bool))


@pytest.mark.parametrize("layout,fuse_silu,pack", [("mlx", False, True), ("pairs", False, True),
                                                   ("pairs", True, True), ("pairs", True, False)])
def test_verify_step_host_path(pkg, monkeypatch, layout, fuse_silu, pack):
    """The benchmark step's host side on CPU, library replaced by a recorder:
    set-up (pair repack, tape recording), the qmm stack, lm_head keys and the
    accept + rollback part all pass the wrappers' argument checks and issue
    the expected launches (two requests' rows share each qmm launch when
    packed: 3 requests -> 2 launches per projection)."""
    import contextlib

    from dflash_mlx_b200 import _lib, kernels, lm_head, verify_qmm, verify_step

    calls = []

    class Recorder:
        def __getattr__(self, name):
            def launch(*args):
                calls.append(name)
                return 0
            return launch

    monkeypatch.setattr(_lib, "load", lambda path=None: Recorder())
    for mod in (verify_qmm, lm_head, kernels, pkg.moe):
        for attr, fake in (("require_cuda", lambda t, name: None), ("stream_ptr", lambda dev: 0),
                           ("workspace", lambda dev, n: torch.zeros(16, dtype=torch.uint8))):
            if hasattr(mod, attr):
                monkeypatch.setattr(mod, attr, fake)
    monkeypatch.setattr(verify_qmm, "workspace_bytes", lambda m, k, n: 16)
    monkeypatch.setattr(lm_head, "workspace_bytes", lambda r, d, v: 16)
    monkeypatch.setattr(torch.cuda, "Stream", lambda dev=None: None)
    monkeypatch.setattr(torch.cuda, "device", lambda dev: contextlib.nullcontext())

    shape = verify_step.StackShape(hidden=256, layers=2, q_out=256, kv_out=128, inter=512, vocab=1000,
                                   gdn_layers=2, gdn_heads=2, gdn_dk=32, gdn_dv=32)
    step = verify_step.VerifyStep("cpu", requests=3, shape=shape, weight_layout=layout,
                                  fuse_silu=fuse_silu, pack_requests=pack)
    setup = list(calls)
    assert setup.count("dfl_gdn_forward_tape") == shape.gdn_layers
    assert setup.count("dfl_repack_w4_pairs") == (4 * shape.layers if layout == "pairs" else 0)
    calls.clear()
    step._qmm_stack()
    per_proj = 2 if pack else 3
    qmm = [c for c in calls if c.startswith("dfl_verify_qmm")]
    assert len(qmm) == per_proj * 4 * shape.layers
    groups = 1 if pack else 3   # the unfused SiLU*up runs once per group of rows
    assert calls.count("dfl_silu_mul_rows_bf16") == (0 if fuse_silu else groups * shape.layers)
    calls.clear()
    step._keys(step.x)
    keys_all = torch.zeros((1, 3 * shape.block), dtype=torch.int64)
    step._accept_and_rollback(keys_all, step.verify_ids)
    assert calls == ["dfl_lmhead_argmax", "dfl_lmhead_accept", "dfl_gdn_tape_replay"]


def test_verify_step_plan_host_path(pkg, monkeypatch):
    """Tiled layout on CPU, library replaced by a recorder: set-up repacks
    every projection once into the tiled layout and encodes one plan whose
    phases are the stack's projections per group of up to eight requests
    (one 128-row token tile), projection-major within a layer (every group's
    q|k|v, then o, gate|up + SiLU, down); the qmm stack is one plan launch."""
    import contextlib

    from dflash_mlx_b200 import _lib, kernels, lm_head, qmm_plan, verify_step

    calls, encoded = [], []

    class Recorder:
        def dfl_w4_tiled_bytes(self, n, k):
            calls.append("dfl_w4_tiled_bytes")
            return ((n + 127) // 128) * ((k + 511) // 512) * 36864

        def dfl_qmm_plan_bytes(self, n):
            return 256 + 192 * n

        def dfl_qmm_plan_encode(self, arr, n, host, nbytes):
            calls.append("dfl_qmm_plan_encode")
            assert nbytes == 256 + 192 * n
            encoded.extend((p.M, p.K, p.N, p.ldx, p.ldy, p.flags, p.dep) for p in arr[:n])
            return 0

        def dfl_qmm_plan_workspace_bytes(self, host, status):
            return 64

        def __getattr__(self, name):
            def launch(*args):
                calls.append(name)
                return 0
            return launch

    monkeypatch.setattr(_lib, "load", lambda path=None: Recorder())
    for mod in (qmm_plan, lm_head, kernels, pkg.moe, pkg.verify_qmm):
        for attr, fake in (("require_cuda", lambda t, name: None), ("stream_ptr", lambda dev: 0),
                           ("workspace", lambda dev, n: torch.zeros(16, dtype=torch.uint8))):
            if hasattr(mod, attr):
                monkeypatch.setattr(mod, attr, fake)
    monkeypatch.setattr(lm_head, "workspace_bytes", lambda r, d, v: 16)
    monkeypatch.setattr(torch.cuda, "Stream", lambda dev=None: None)
    monkeypatch.setattr(torch.cuda, "device", lambda dev: contextlib.nullcontext())

    shape = verify_step.StackShape(hidden=256, layers=2, q_out=256, kv_out=128, inter=512, vocab=1000,
                                   gdn_layers=2, gdn_heads=2, gdn_dk=32, gdn_dv=32)
    with pytest.raises(ValueError):
        verify_step.VerifyStep("cpu", requests=1, shape=shape, weight_layout="tiled", fuse_silu=False)
    calls.clear()
    encoded.clear()
    step = verify_step.VerifyStep("cpu", requests=10, shape=shape, weight_layout="tiled", fuse_silu=True)
    assert calls.count("dfl_repack_w4_tiled") == 4 * shape.layers
    assert calls.count("dfl_qmm_plan_encode") == 1
    assert step.layers is None and len(step.tiled) == shape.layers
    h, q_n, inter = shape.hidden, shape.q_out + 2 * shape.kv_out, shape.inter
    want = []
    last = {0: -1, 1: -1}
    rows = ((0, 128), (1, 32))            # 10 requests: rows 0-127 and 128-159
    for _ in range(shape.layers):
        # projection-major inside a layer: every group's q|k|v, o, gate|up, down;
        # dataflow: q|k|v waits for the group's previous down (its input),
        # down for the group's gate|up SiLU output; o and gate|up read stand-ins
        base = len(want)
        want += [(m, h, q_n, h, q_n, 2, last[g]) for g, m in rows]
        want += [(m, shape.q_out, h, shape.q_out, h, 2, -1) for g, m in rows]
        want += [(m, h, 2 * inter, h, inter, 3, -1) for g, m in rows]
        want += [(m, inter, h, inter, h, 2, base + 4 + g) for g, m in rows]
        for g, _ in rows:
            last[g] = base + 6 + g
    assert encoded == want
    # the chained form: o, gate|up and down also wait for the group's previous
    # projection (two phases back in the projection-major order)
    encoded.clear()
    step._build_plan("chain")
    assert [e[-1] for e in encoded] == [w[-1] if (i % 8) < 2 else i - 2 for i, w in enumerate(want)]
    calls.clear()
    step._qmm_stack()
    assert calls == ["dfl_qmm_plan_run"]
