"""The C-ABI library loads on a CPU-only machine and exports every symbol include/wisp_b200.h declares;
the host-only entry points work without a GPU."""

import ctypes
import os
import re

import pytest

from oracle import wisp_oracle as O
from wisp import _lib

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "wisp_b200.h")


def declared():
    src = open(HEADER).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return sorted(set(re.findall(r"\b(wisp_\w+)\s*\(", src)))


def test_header_matches_binding_table():
    assert declared() == sorted(_lib.SIGNATURES)


def test_library_exports_every_declared_symbol():
    L = ctypes.CDLL(_lib.LIB_PATH)
    missing = [s for s in declared() if not hasattr(L, s)]
    assert not missing, missing


def test_version_and_error_string():
    L = _lib.lib()
    assert L.wisp_version() >= 100
    assert isinstance(L.wisp_last_error(), bytes)


@pytest.mark.parametrize("bits", [16, 8, 4, 3, 2])
@pytest.mark.parametrize("n,group", [(1572864, 128), (2048, 32), (32768, 128), (4096, 64)])
def test_expert_nbytes_matches_oracle(bits, n, group):
    assert _lib.lib().wisp_expert_nbytes(n, bits, group) == O.expert_nbytes(n, bits, group)


def test_expert_nbytes_rejects_bad_shapes():
    L = _lib.lib()
    assert L.wisp_expert_nbytes(1000, 4, 128) == -1  # 3n not divisible by the group
    assert L.wisp_expert_nbytes(2048, 5, 128) == -1  # unsupported bit width
    assert L.wisp_expert_nbytes(0, 4, 128) == -1


def test_invalid_arguments_fail_on_host_without_a_gpu():
    """Argument checks run before any launch, so they report cleanly even on a CPU-only machine."""
    L = _lib.lib()
    rc = L.wisp_moe_decode(None, 8, 2506752, None, 8, None, 2048, 768, 4, 128, None, 0, None, None)
    assert rc == _lib.WISP_ERR_INVALID
    assert b"NULL" in L.wisp_last_error()
    with pytest.raises(_lib.WispError, match="bits must be"):
        _lib.call("wisp_moe_decode", 16, 8, 2506752, 16, 8, 16, 2048, 768, 5, 128, 16, 8 * 768, 16, None)


def test_gptoss_alignment_checks_run_on_host():
    """The gpt-oss entry point rejects an output or bias pointer that is not 8-byte aligned (its
    reductions store and load 8-byte vectors) before touching the device."""
    from oracle import wisp_oracle as O

    H = I = 256
    nb = O.expert_nbytes(H * I, 4, 128)
    args = dict(pool=4096, nslots=8, nbytes=nb, meta=4096, experts=4096, N=1, k=2, x=4096, H=H, I=I, bits=4, group=128,
                gub=4096, db=4096, ws=4096, wsb=1 << 30, out=4096, stream=None)

    def call(**kw):
        a = dict(args, **kw)
        return _lib.call("wisp_moe_gptoss", a["pool"], a["nslots"], a["nbytes"], a["meta"], a["experts"], a["N"], a["k"],
                         a["x"], a["H"], a["I"], a["bits"], a["group"], a["gub"], a["db"], a["ws"], a["wsb"], a["out"],
                         a["stream"])

    for bad in (dict(out=4098), dict(gub=4100), dict(db=4102)):
        with pytest.raises(_lib.WispError, match="8-byte aligned"):
            call(**bad)
    with pytest.raises(_lib.WispError, match="16-byte aligned"):
        call(x=4104)
