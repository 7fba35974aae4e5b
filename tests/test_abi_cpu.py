"""The C ABI library on a machine without a GPU: it loads, exports every
entry point include/trs.h declares, and its host-side planning (broadcasting,
view validation, dimension folding, kernel choice) behaves as designed.  No
call here launches a kernel."""
from __future__ import annotations

import ctypes
import re

import pytest

from conftest import ROOT


def declared_entry_points() -> list[str]:
    text = (ROOT / "include" / "trs.h").read_text()
    return sorted(set(re.findall(r"^\s*(?:trs_status|int32_t|size_t|uint64_t|const char\*)\s+(trs_[a-z0-9_]+)\(",
                                 text, flags=re.M)))


def test_library_exports_every_declared_entry_point(trs):
    lib = trs.load()
    names = declared_entry_points()
    assert len(names) >= 30
    for n in names:
        assert hasattr(lib, n), n
    assert set(names) == set(trs.exported_names())


def test_abi_version(trs):
    assert trs.load().trs_abi_version() == 1


def _bcast(trs, a, b):
    lib = trs.load()
    out = (ctypes.c_int64 * 8)()
    nd = ctypes.c_int32()
    st = lib.trs_broadcast_shape((ctypes.c_int64 * 8)(*a), len(a), (ctypes.c_int64 * 8)(*b), len(b), out,
                                 ctypes.byref(nd))
    return st, [out[i] for i in range(nd.value)]


@pytest.mark.parametrize("a,b,want", [
    ([4], [1], [4]), ([2, 3], [1, 3], [2, 3]), ([2, 3], [3], [2, 3]),
    ([64, 256, 56, 56], [1, 256, 1, 1], [64, 256, 56, 56]), ([1], [5, 1, 7], [5, 1, 7]),
    ([8, 1, 6, 1], [7, 1, 5], [8, 7, 6, 5]),
])
def test_broadcast_shape_matches_reference_rules(trs, a, b, want):
    st, got = _bcast(trs, a, b)
    assert st == trs.OK and got == want


def test_broadcast_shape_incompatible(trs):
    st, _ = _bcast(trs, [2, 3], [2])
    assert st == trs.ERR_SHAPE
    assert "incompatible shapes" in trs.last_error()


def _plan(trs, prog, ins, out):
    lib = trs.load()
    variant, nd, vw = ctypes.c_int32(), ctypes.c_int32(), ctypes.c_int32()
    shp = (ctypes.c_int64 * 8)()
    strides = (ctypes.c_int64 * 32)()
    st = lib.trs_plan_elementwise(ctypes.byref(prog), trs.views_array(ins), ctypes.byref(out) if out else None,
                                  ctypes.byref(variant), ctypes.byref(nd), shp, strides, ctypes.byref(vw))
    trs.check(st)
    n = nd.value
    return variant.value, [shp[i] for i in range(n)], [[strides[k * 8 + i] for i in range(n)] for k in range(4)], vw.value


BASE = 1 << 20  # a 16-byte aligned fake device address; planning never dereferences it


def test_plan_row_bias_add_folds_to_two_dims_vector_kernel(trs):
    # config 1: A[1024,1024] + b[1024]
    a = trs.make_view(BASE, trs.F32, [1024, 1024])
    b = trs.make_view(BASE + (1 << 24), trs.F32, [1024])
    out = trs.make_view(BASE + (1 << 26), trs.F32, [1024, 1024])
    var, shape, st, vw = _plan(trs, trs.program(2, trs.ADD), [a, b], out)
    assert var == 0 and vw == 4
    assert shape == [1024, 1024]
    assert st[2] == [0, 1]


def test_plan_same_shape_contiguous_folds_to_one_dim(trs):
    a = trs.make_view(BASE, trs.F32, [64, 32, 16])
    b = trs.make_view(BASE + (1 << 24), trs.F32, [64, 32, 16])
    out = trs.make_view(BASE + (1 << 26), trs.F32, [64, 32, 16])
    var, shape, st, vw = _plan(trs, trs.program(2, trs.MUL), [a, b], out)
    assert var == 0 and shape == [64 * 32 * 16] and vw == 4


def test_plan_transposed_operand_uses_tile_kernel(trs):
    # config 2: A[4096,4096] & B^T with B^T strides [1, 4096]
    a = trs.make_view(BASE, trs.F32, [4096, 4096])
    bt = trs.make_view(BASE + (1 << 27), trs.F32, [4096, 4096], [1, 4096])
    out = trs.make_view(BASE + (1 << 28), trs.F32, [4096, 4096])
    var, shape, st, _ = _plan(trs, trs.program(2, trs.MUL, epilogue="sigmoid"), [a, bt], out)
    assert var == 1
    assert st[2] == [1, 4096]


def test_plan_nchw_channel_broadcast(trs):
    # config 4: X[64,256,56,56] & s[1,256,1,1] + b[1,256,1,1]: H,W fold into one run
    x = trs.make_view(BASE, trs.F32, [64, 256, 56, 56])
    s = trs.make_view(BASE + (1 << 30), trs.F32, [1, 256, 1, 1])
    b = trs.make_view(BASE + (1 << 30) + 4096, trs.F32, [1, 256, 1, 1])
    out = trs.make_view(BASE + (1 << 31), trs.F32, [64, 256, 56, 56])
    var, shape, st, vw = _plan(trs, trs.program(3, trs.MUL, trs.ADD, "relu"), [x, s, b], out)
    assert var == 0 and vw == 4
    assert shape == [64, 256, 3136]
    assert st[2] == [0, 1, 0] and st[3] == [0, 1, 0]


def test_plan_reversed_view_uses_generic_kernel(trs):
    a = trs.make_view(BASE, trs.F32, [100], [-1], 99)
    out = trs.make_view(BASE + 4096, trs.F32, [100])
    var, _, _, _ = _plan(trs, trs.program(1), [a], out)
    assert var == 2


def test_plan_unaligned_offset_falls_back_to_scalar_width(trs):
    a = trs.make_view(BASE, trs.F32, [1024], None, 1, storage_len=1025)
    out = trs.make_view(BASE + 8192, trs.F32, [1024])
    var, _, _, vw = _plan(trs, trs.program(1), [a], out)
    assert var == 0 and vw == 1


def test_view_outside_its_storage_is_rejected(trs):
    a = trs.make_view(BASE, trs.F32, [10, 10], storage_len=99)
    out = trs.make_view(BASE + 8192, trs.F32, [10, 10])
    with pytest.raises(trs.TrsError) as e:
        _plan(trs, trs.program(1), [a], out)
    assert e.value.status == trs.ERR_VIEW


def test_negative_stride_below_zero_is_rejected(trs):
    a = trs.make_view(BASE, trs.F32, [10], [-1], 5, storage_len=10)
    out = trs.make_view(BASE + 8192, trs.F32, [10])
    with pytest.raises(trs.TrsError) as e:
        _plan(trs, trs.program(1), [a], out)
    assert e.value.status == trs.ERR_VIEW


def test_output_must_have_broadcast_shape(trs):
    a = trs.make_view(BASE, trs.F32, [2, 3])
    b = trs.make_view(BASE + 4096, trs.F32, [3])
    out = trs.make_view(BASE + 8192, trs.F32, [3, 2])
    with pytest.raises(trs.TrsError) as e:
        _plan(trs, trs.program(2, trs.ADD), [a, b], out)
    assert e.value.status == trs.ERR_SHAPE


def test_incompatible_shapes_give_the_reference_message(trs):
    a = trs.make_view(BASE, trs.F32, [2, 3])
    b = trs.make_view(BASE + 4096, trs.F32, [2])
    out = trs.make_view(BASE + 8192, trs.F32, [2, 3])
    with pytest.raises(trs.TrsError) as e:
        _plan(trs, trs.program(2, trs.MUL), [a, b], out)
    assert "!!!MulElems: incompatible shapes!!!" in e.value.message


def test_output_aliasing_an_input_through_another_layout_is_rejected(trs):
    a = trs.make_view(BASE, trs.F32, [64, 64])
    at = trs.make_view(BASE, trs.F32, [64, 64], [1, 64])
    with pytest.raises(trs.TrsError) as e:
        _plan(trs, trs.program(2, trs.ADD), [a, at], a)
    assert e.value.status == trs.ERR_ALIAS


def test_in_place_on_identical_layout_is_allowed(trs):
    a = trs.make_view(BASE, trs.F32, [64, 64])
    b = trs.make_view(BASE + (1 << 20), trs.F32, [64, 64])
    var, _, _, _ = _plan(trs, trs.program(2, trs.ADD), [a, b], a)
    assert var == 0


def test_transcendental_on_integers_is_rejected(trs):
    a = trs.make_view(BASE, trs.I32, [8])
    out = trs.make_view(BASE + 4096, trs.I32, [8])
    with pytest.raises(trs.TrsError) as e:
        _plan(trs, trs.program(1, epilogue="sigmoid"), [a], out)
    assert e.value.status == trs.ERR_DTYPE
