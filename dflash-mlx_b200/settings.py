"""Environment settings of the verify path.

The variable names and their meaning are the reference's (a drop-in reads the
same switches); the code is this package's own.  Read once per call of
:func:`read`, so a test can change the environment between calls.

=========================  ==================================================
``DFLASH_VERIFY_LINEAR``   "1" / "0" force the verify linears on / off; unset
                           leaves the choice to the caller
``DFLASH_VERIFY_QMM``      "1" reports the verify qmm as enabled
                           (``verify_qmm.is_enabled``); on B200 the sm_100a
                           kernel is the only implementation, so it selects
                           nothing
``DFLASH_VERIFY_MAX_N``    linears with at least this many output features
                           stay ineligible (default 100000)
``DFLASH_VERIFY_INCLUDE``  comma list of path tags (or ``mlp`` / ``attn`` /
                           ``gdn`` groups) that may be swapped; ``all`` or
                           empty = every tag
=========================  ==================================================

The reference's kernel-variant and split-K switches select Metal kernels;
the sm_100a kernel chooses its split itself (stream-K), so they have no
counterpart here and are not read.
"""

from __future__ import annotations

import os
from dataclasses import dataclass
from typing import FrozenSet, Optional

MAX_N_DEFAULT = 100_000

_GROUPS = {
    "mlp": ("mlp_gate", "mlp_up", "mlp_down"),
    "attn": ("attn_q", "attn_k", "attn_v", "attn_o"),
    "gdn": ("gdn_qkv", "gdn_z", "gdn_o"),
}


@dataclass(frozen=True)
class VerifySettings:
    linear: Optional[bool]          # forced on / off, or None
    qmm: bool
    max_n: int
    include: Optional[FrozenSet[str]]  # None = every path tag

    def allows(self, tag: str) -> bool:
        return self.include is None or tag in self.include


def _int(name: str, default: int) -> int:
    raw = os.environ.get(name)
    if raw is None:
        return default
    try:
        return int(raw)
    except ValueError:
        return default


def read() -> VerifySettings:
    lin = os.environ.get("DFLASH_VERIFY_LINEAR", "").strip()
    linear = {"1": True, "0": False}.get(lin)
    spec = os.environ.get("DFLASH_VERIFY_INCLUDE", "all").strip().lower()
    include = None
    if spec not in ("", "all"):
        tags = set()
        for item in (s.strip() for s in spec.split(",")):
            if item:
                tags.add(item)
                tags.update(_GROUPS.get(item, ()))
        include = frozenset(tags)
    return VerifySettings(linear=linear,
                          qmm=os.environ.get("DFLASH_VERIFY_QMM", "") == "1",
                          max_n=_int("DFLASH_VERIFY_MAX_N", MAX_N_DEFAULT),
                          include=include)
