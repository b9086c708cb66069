"""The C ABI without a GPU: the library loads, exports every entry point include/ptsim_b200.h declares,
agrees with the Python mirror of ptsim_desc, and validates descriptors on the host (ptsim_check), refusing
malformed ones and index maps that would leave their tensors -- the host side of the GPU's bounds checks
(the reference maps such accesses to its INVALID_SPAD_ACCESS trap, runtime/spike.py:12)."""
import ctypes
import os
import re

import pytest

from pytorchsim_triton_compiler.codegen import build as B
from pytorchsim_triton_compiler.codegen import descriptors as D
from pytorchsim_triton_compiler.contract import kernel_object as ko
from pytorchsim_triton_compiler.runtime import native

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "ptsim_b200.h")


def declared():
    text = open(HEADER).read()
    return sorted(set(re.findall(r"^\w[\w\s\*]*?\b(ptsim_\w+)\(", text, flags=re.M)))


def test_library_exports_every_declared_symbol():
    lib = native.load()
    names = declared()
    assert names, "no declarations found in the header"
    assert set(names) == set(native.SYMBOLS), (names, sorted(native.SYMBOLS))
    raw = ctypes.CDLL(native.library_path())
    for n in names:
        assert hasattr(raw, n), n
    assert lib.ptsim_version() == D.ABI_VERSION
    assert lib.ptsim_desc_size() == D.SIZE


def test_fixture_descriptors_validate():
    objs = os.path.join(ROOT, "tests", "golden", "objects")
    n = 0
    for name in sorted(os.listdir(objs)):
        m = ko.read(os.path.join(objs, name))
        blob = ko.read_desc(os.path.join(objs, name), m)
        native.check(blob)
        assert native.units(blob) == D.from_bytes(blob).units
        n += 1
    assert n >= 40


def _code(fn):
    with pytest.raises(native.ExecutorError) as e:
        fn()
    return e.value.code


def test_malformed_descriptors_are_refused():
    good = B.row_softmax(64, 256)
    native.check(D.to_bytes(good))
    bad = B.row_softmax(64, 256)
    bad.magic = 0x12345678
    assert _code(lambda: native.check(D.to_bytes(bad))) == D.E_DESC
    bad = B.row_softmax(64, 256)
    bad.version = 99
    assert _code(lambda: native.check(D.to_bytes(bad))) == D.E_DESC
    bad = B.row_softmax(64, 256)
    bad.kind = 42
    assert _code(lambda: native.check(D.to_bytes(bad))) == D.E_DESC
    assert _code(lambda: native.check(D.to_bytes(good)[:100])) == D.E_DESC


def test_out_of_bounds_maps_are_refused_on_the_host():
    # A copy whose source map reaches one element past its tensor.
    d = B.copy_map(1000, 1000, [(1, 1000, 1)])
    d.p.ew.map[0].offset = 1
    assert _code(lambda: native.check(D.to_bytes(d))) == D.E_OOB
    # Rows past the tensor.
    d = B.row_softmax(64, 256)
    d.p.row.rows = 65
    assert _code(lambda: native.check(D.to_bytes(d))) == D.E_OOB
    # GEMM operands larger than their tensors.
    d = B.gemm(128, 256, 64)
    d.p.gemm.K = 128
    assert _code(lambda: native.check(D.to_bytes(d))) == D.E_OOB


def test_launch_refuses_bad_ranges_and_pointer_counts_without_touching_a_gpu():
    blob = D.to_bytes(B.row_softmax(64, 256))
    assert _code(lambda: native.launch(blob, [1], 0, 1)) == D.E_ARGS          # 1 pointer for 2 arguments
    assert _code(lambda: native.launch(blob, [1, 2], 0, 99)) == D.E_ARGS      # past the units
    assert _code(lambda: native.launch(blob, [0, 2], 0, 1)) == D.E_ARGS       # a null pointer


def test_descriptor_round_trip():
    d = B.gemm(256, 512, 128, residual=True)
    blob = D.to_bytes(d)
    e = D.from_bytes(blob)
    assert (e.kind, e.p.gemm.M, e.p.gemm.N, e.p.gemm.K, e.p.gemm.r_arg) == (D.GEMM, 256, 512, 128, 0)
    assert D.describe(e)["residual"] is True


def test_fused_and_routing_descriptors_are_checked_on_the_host():
    """The newer descriptor fields: fused vector programs, integer tables, the fused combine, the residual
    RMSNorm row -- valid ones pass ptsim_check, malformed ones are refused with their code."""
    for good in (B.rmsnorm_gemv(4096, 4096), B.silu_gemv(4096, 12288), B.sumsq(4096, True), B.expert_counts(1024, 128),
                 B.slot_of(1024, 128), B.group_tables(128), B.count_le(128, 128), B.cumsum_int(128, "int32", "int32"),
                 B.combine_gather_sum(128, 2048, 8, 128, fused=True)):
        native.check(D.to_bytes(good))
    # a vector program with an opcode past the elementwise set, a register past r7, a load slot it lacks
    for field, value in (("op", 99), ("dst", 8), ("a", 3)):
        d = B.rmsnorm_gemv(256, 256)
        setattr(d.p.gemm.pro.code[0], field, value)
        assert _code(lambda: native.check(D.to_bytes(d))) == D.E_DESC, field
    # a fused program on a GEMM of M > 1
    d = B.rmsnorm_gemv(256, 256)
    d.p.gemm.M = 2
    assert _code(lambda: native.check(D.to_bytes(d))) in (D.E_DESC, D.E_OOB)
    # an integer table storing into a float tensor, an output past the table, an unknown instruction
    d = B.expert_counts(64, 8)
    d.arg_dtype[1] = D.DTYPE_CODE["float32"]
    assert _code(lambda: native.check(D.to_bytes(d))) == D.E_UNSUPPORTED
    d = B.expert_counts(64, 8)
    d.p.itab.nout = 5
    assert _code(lambda: native.check(D.to_bytes(d))) == D.E_DESC
    d = B.expert_counts(64, 8)
    d.p.itab.code[0].op = 40
    assert _code(lambda: native.check(D.to_bytes(d))) == D.E_DESC
    # a combine with three residual rows; a residual RMSNorm whose residual tensor is too short
    d = B.combine_gather_sum(16, 64, 2, 4, fused=True)
    d.p.gsum.nres = 3
    assert _code(lambda: native.check(D.to_bytes(d))) == D.E_DESC
    d = B.row_rmsnorm(64, 256)
    d.p.row.res_arg_p1 = 1        # the residual is argument 0: the input itself, as long as the rows -- valid
    native.check(D.to_bytes(d))
    d.p.row.rows = 64
    d.arg_numel[0] = 64 * 256 - 1
    assert _code(lambda: native.check(D.to_bytes(d))) == D.E_OOB
