"""The C-ABI library: loads without a GPU, exports every declared symbol, and
rejects bad arguments on the host before touching the device."""
import ctypes
import os
import re

import pytest

from fastaf_kernel_b200 import _lib
from fastaf_kernel_b200.build import INCLUDE, LIB_PATH

HEADER = os.path.join(INCLUDE, "gdn_b200.h")


def declared_symbols():
    text = open(HEADER).read()
    return sorted(set(re.findall(r"GDN_API\s+[\w\s\*]*?\b(gdn_\w+)\s*\(", text)))


def test_library_built_in_tree():
    assert os.path.exists(LIB_PATH), "run __graft_entry__.build() first"


def test_header_declares_the_bound_symbols():
    assert declared_symbols() == sorted(_lib.EXPORTED_SYMBOLS)


def test_every_declared_symbol_is_exported():
    lib = ctypes.CDLL(LIB_PATH)
    for name in declared_symbols():
        assert hasattr(lib, name), name


def test_version():
    assert _lib.version().startswith("gdn_b200")


def _decode(lib, **over):
    args = dict(q=16, k=16, v=16, state=16, A_log=16, a=16, dt_bias=16, b=16, batch=1,
                Hq=16, Hv=32, D=128, scale=0.0, gd=1, pd=0, out=16, ns=16, stream=None)
    args.update(over)
    return lib.gdn_decode(args["q"], args["k"], args["v"], args["state"], args["A_log"],
                          args["a"], args["dt_bias"], args["b"], args["batch"], args["Hq"],
                          args["Hv"], args["D"], args["scale"], args["gd"], args["pd"],
                          args["out"], args["ns"], args["stream"])


def _prefill(lib, method=0, **over):
    args = dict(q=16, k=16, v=16, state=None, A_log=16, a=16, dt_bias=16, b=16, cu=16, N=1,
                T=4, Hq=16, Hv=32, D=128, scale=0.0, gd=1, pd=0, out=16, ns=4096)
    args.update(over)
    return lib.gdn_prefill_ex(args["q"], args["k"], args["v"], args["state"], args["A_log"],
                              args["a"], args["dt_bias"], args["b"], args["cu"], args["N"],
                              args["T"], args["Hq"], args["Hv"], args["D"], args["scale"],
                              args["gd"], args["pd"], args["out"], args["ns"], method, None)


@pytest.mark.parametrize("over,code", [
    (dict(D=64), _lib.GDN_ERR_UNSUPPORTED),
    (dict(Hv=24, Hq=16), _lib.GDN_ERR_INVALID_ARGUMENT),
    (dict(Hq=0), _lib.GDN_ERR_INVALID_ARGUMENT),
    (dict(gd=7), _lib.GDN_ERR_INVALID_ARGUMENT),
    (dict(q=None), _lib.GDN_ERR_INVALID_ARGUMENT),
    (dict(q=8), _lib.GDN_ERR_INVALID_ARGUMENT),               # misaligned
    (dict(batch=-1), _lib.GDN_ERR_INVALID_ARGUMENT),
    (dict(state=16, ns=32), _lib.GDN_ERR_INVALID_ARGUMENT),   # partial overlap
])
def test_decode_rejects_bad_arguments(over, code):
    lib = _lib.load()
    assert _decode(lib, **over) == code
    assert lib.gdn_last_error().decode()


def test_decode_empty_batch_is_a_noop():
    assert _decode(_lib.load(), batch=0) == _lib.GDN_OK


@pytest.mark.parametrize("over,code", [
    (dict(D=256), _lib.GDN_ERR_UNSUPPORTED),
    (dict(cu=None), _lib.GDN_ERR_INVALID_ARGUMENT),
    (dict(N=-1), _lib.GDN_ERR_INVALID_ARGUMENT),
    (dict(T=1 << 31), _lib.GDN_ERR_INVALID_ARGUMENT),
    (dict(state=16, ns=16), _lib.GDN_ERR_INVALID_ARGUMENT),  # prefill never aliases
])
def test_prefill_rejects_bad_arguments(over, code):
    lib = _lib.load()
    assert _prefill(lib, **over) == code
    assert lib.gdn_last_error().decode()


def test_prefill_rejects_unknown_method():
    assert _prefill(_lib.load(), method=9) == _lib.GDN_ERR_INVALID_ARGUMENT


def test_prefill_no_sequences_is_a_noop():
    assert _prefill(_lib.load(), N=0, T=0) == _lib.GDN_OK


def test_error_maps_to_python_exceptions():
    lib = _lib.load()
    with pytest.raises(NotImplementedError):
        _lib.check(_decode(lib, D=64))
    with pytest.raises(ValueError):
        _lib.check(_decode(lib, q=None))


@pytest.mark.parametrize("n,hq,hv,sms,launches", [
    (16, 16, 32, 148, 5),    # 512 chains: the last 68 go to the second stream; sequences ranked
    (4, 16, 32, 148, 2),     # fewer chains than SMs: no split, no ranking
    (37, 2, 4, 148, 2),      # 148 chains: whole waves, no split, not more chains than SMs
    (74, 2, 4, 148, 3),      # 296 chains: whole waves, no split; sequences ranked
    (13, 4, 12, 148, 5),     # one v-head per prep CTA: tail of 8; sequences ranked
    (16, 16, 32, 147, 3),    # a tail of 71 is not a whole number of two-head prep CTAs
    (1, 4, 512, 148, 4),     # one sequence of 512 chains: a tail of 68 split off, nothing to rank
    (65537, 2, 4, 148, 4),   # more sequences than are ranked: index order (tail of 40 split off)
    (1, 3, 4, 148, 0),       # invalid head counts
])
def test_prefill_tc_launch_count_rule(n, hq, hv, sms, launches):
    """The host query of the tcgen05 prefill's launch count: the wave-split rule, plus
    the ranking of the sequences when there are several and more chains than SMs."""
    assert _lib.load().gdn_prefill_tc_launches(n, hq, hv, sms) == launches
