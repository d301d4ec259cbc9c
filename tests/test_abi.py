"""The C-ABI library loads, exports every symbol include/amoe.h declares, and
validates configurations on the host (no GPU needed for any of this)."""
import ctypes
import os
import re

import pytest

from airllm_b200 import moe

HEADER = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "include", "amoe.h")


def declared_symbols():
    text = open(HEADER).read()
    return sorted(set(re.findall(r"AMOE_API\s+[\w\s\*]+?\b(amoe_\w+)\s*\(", text)))


def test_header_declares_the_binding_table():
    assert declared_symbols() == sorted(moe.SIGNATURES)


def test_library_exports_every_declared_symbol():
    lib = moe.load_library()
    for name in declared_symbols():
        assert hasattr(lib, name), name
    assert lib.amoe_abi_version() == 1


def _cfg(**kw):
    base = dict(hidden=2880, intermediate=2880, experts=32, top_k=4, layers=1, rms_eps=1e-5,
                swiglu_alpha=1.702, swiglu_limit=7.0, max_tokens=16, device=0, stream_slots=0,
                ep_size=1, ep_rank=0, nccl_id=None, path=0)
    base.update(kw)
    return moe.AmoeConfig(**base)


@pytest.mark.parametrize("bad,msg", [
    (dict(hidden=2880 + 32), "hidden"),
    (dict(intermediate=0), "intermediate"),
    (dict(experts=0), "experts"),
    (dict(top_k=33, experts=64), "top-k"),
    (dict(top_k=5, experts=4), "top-k"),
    (dict(rms_eps=0.0), "epsilon"),
    (dict(swiglu_alpha=1.5), "swiglu"),
    (dict(max_tokens=0), "max_tokens"),
    (dict(stream_slots=1), "stream_slots"),
    (dict(stream_experts=1), "stream_experts"),
    (dict(stream_slots=2, path=1), "stream_slots needs path"),
    (dict(ep_rank=2, ep_size=2), "ep_rank"),
    (dict(path=7), "path"),
])
def test_create_rejects_invalid_configs_without_touching_the_gpu(bad, msg):
    lib = moe.load_library()
    h = ctypes.c_void_p()
    rc = lib.amoe_create(ctypes.byref(_cfg(**bad)), ctypes.byref(h))
    assert rc == moe.AMOE_ERR_INVALID
    assert not h.value
    assert msg in lib.amoe_last_error(None).decode()


def test_null_context_calls_fail_cleanly():
    lib = moe.load_library()
    assert lib.amoe_forward(None, 0, None, 1, None, None, None) == moe.AMOE_ERR_INVALID
    assert lib.amoe_synchronize(None) == moe.AMOE_ERR_INVALID
    lib.amoe_destroy(None)  # no-op
