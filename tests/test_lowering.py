"""The B200 lowering (targets/b200): the reference's own kernels lower to the committed descriptors (when
the reference tree is present), kernels written for this suite lower to the expected classes and index
maps, and programs outside the executor's classes are refused with a Reason, never approximated."""
import json
import os

import pytest

from pytorchsim_triton_compiler.codegen import descriptors as D
from pytorchsim_triton_compiler.contract import kernel_object as ko
from pytorchsim_triton_compiler.contract.kernel_spec import load_spec
from pytorchsim_triton_compiler.contract.stop import Reason, Refused
from pytorchsim_triton_compiler.targets.b200 import frontend as F
from pytorchsim_triton_compiler.targets.b200 import lower as L

HERE = os.path.dirname(os.path.abspath(__file__))
REF = os.environ.get("PTSIM_REFERENCE", "")   # the reference checkout, when a caller provides one
OBJ = os.path.join(HERE, "golden", "objects")


def test_index_algebra():
    x = F.Index.var("x")
    e = x.mod(128) + x.floordiv(262144).scale(128) + x.floordiv(128).mod(2048).scale(1024)
    assert e.terms == {F.Digit("x", 1, 128): 1, F.Digit("x", 262144, None): 128, F.Digit("x", 128, 2048): 1024}
    with pytest.raises(Refused):
        (x + 1).floordiv(4)
    with pytest.raises(Refused):
        x.floordiv(128).mod(2048).floordiv(3)


def test_own_pointwise_kernel_lowers_to_its_dma_boxes():
    spec = load_spec(os.path.join(HERE, "kernels", "relayout_scale.py"))
    lo = L.lower(spec)
    d = lo.desc
    assert d.kind == D.ELEMENTWISE and d.units == 4 and d.unit_size == 2048
    maps = {m.arg: sorted((m.div[k], m.mod[k], m.stride[k]) for k in range(m.ndigit)) for m in list(d.p.ew.map)[:d.p.ew.nmap]}
    assert maps[0] == [(1, 32, 1), (32, 4, 2048), (128, 64, 32)]
    assert maps[1] == [(1, 8192, 1)] and maps[2] == [(1, 8192, 1)]
    ops = [D.OP_NAME[i.op] for i in list(d.p.ew.code)[:d.p.ew.ncode]]
    assert ops.count("load") == 2 and "mul" in ops and "add" in ops and ops[-1] == "store"


def test_own_softmax_kernel_is_a_row_program():
    spec = load_spec(os.path.join(HERE, "kernels", "row_softmax.py"))
    lo = L.lower(spec)
    r = lo.desc.p.row
    assert lo.desc.kind == D.ROW_SOFTMAX and (r.rows, r.cols, r.in_row_stride, r.out_row_stride) == (256, 512, 512, 512)
    assert lo.desc.units == 16 and lo.desc.unit_size == 16


def test_atomics_are_refused():
    spec = load_spec(os.path.join(HERE, "kernels", "atomic_accumulate.py"))
    with pytest.raises(Refused) as e:
        L.lower(spec)
    assert e.value.reason == spec.expect_stop.reason


def fixture_names():
    with open(os.path.join(HERE, "golden", "index.json")) as fh:
        return json.load(fh)


@pytest.mark.skipif(not REF or not os.path.isdir(REF), reason="PTSIM_REFERENCE does not name a reference checkout")
@pytest.mark.parametrize("name", [n for n in fixture_names() if "t2048" not in n and "4096x4096" not in n
                                  and "8192" not in n and "b4" not in n and "1m" not in n])
def test_reference_kernels_lower_to_the_committed_descriptors(name):
    d = os.path.join(OBJ, name)
    case = json.load(open(os.path.join(d, "case.json")))
    if case.get("modified"):
        pytest.skip("lowered from a resized copy of the reference's spec")
    spec = load_spec(os.path.join(REF, case["source"]))
    lo = L.lower(spec)
    assert lo.blob == ko.read_desc(d), name


@pytest.mark.skipif(not REF or not os.path.isdir(REF), reason="PTSIM_REFERENCE does not name a reference checkout")
def test_every_decode_and_m1_workload_lowers():
    """All attention_decode_* (28) and gemm_1x* (13) workloads of the bundle lower: decode to one unit per KV
    head with the program's G, S and BKV; the M = 1 matmul (a multiply-reduce program) to a GEMM descriptor
    with M = 1, N = xnumel and K = r0_numel over the N-contiguous matrix."""
    base = os.path.join(REF, "validation", "pytorchsim")
    seen = {"decode": 0, "gemv": 0}
    for wl in sorted(os.listdir(base)):
        if not (wl.startswith("attention_decode_") or wl.startswith("gemm_1x")):
            continue
        kd = os.path.join(base, wl, next(n for n in sorted(os.listdir(os.path.join(base, wl))) if n.startswith("00_")))
        spec = load_spec(os.path.join(kd, next(f for f in os.listdir(kd) if f.endswith("_spec.py"))))
        desc = D.from_bytes(L.lower(spec).blob)
        if wl.startswith("attention_decode_"):
            hq, hkv, s = (int(v) for v in wl.split("_")[2].split("x"))
            a = desc.p.attn
            assert desc.kind == D.ATTN_DECODE and desc.units == hkv == a.hkv, wl
            assert (a.hq, a.seq, a.dim, a.ref_bq, a.ref_bkv) == (hq, s, 128, 16, s), wl
            seen["decode"] += 1
        else:
            k, n = (int(v) for v in wl.split("_")[1].split("x")[1:3])
            g = desc.p.gemm
            assert desc.kind == D.GEMM and (g.M, g.N, g.K, g.b_kmajor, g.ldb) == (1, n, k, 0, n), wl
            seen["gemv"] += 1
    assert seen == {"decode": 28, "gemv": 13}


def test_routing_table_builders_match_the_lowered_objects():
    """The INT_TABLE builders (codegen/build.py) state the same descriptors the lowering made from the
    reference's kernels (layer_op_combine_*/00-02, layer_op_gmm_*/01-03)."""
    import os
    from pytorchsim_triton_compiler.codegen import build as B
    from pytorchsim_triton_compiler.codegen import descriptors as D
    from pytorchsim_triton_compiler.contract import kernel_object as ko
    obj = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "objects")
    pairs = [("moe_combine_t128_00_counts", B.expert_counts(1024, 128)), ("moe_combine_01_offsets", B.cumsum_int(128)),
             ("moe_gmm_01_offsets", B.cumsum_int(128, "int32", "int32")),
             ("moe_combine_t128_02_slot", B.slot_of(1024, 128)), ("moe_gmm_02_group_tables", B.group_tables(128)),
             ("moe_gmm_03_count_le", B.count_le(128, 128)), ("moe_combine_t4096_00_counts", B.expert_counts(32768, 128))]
    for name, d in pairs:
        m = ko.read(os.path.join(obj, name))
        ref = D.from_bytes(ko.read_desc(os.path.join(obj, name), m))
        assert bytes(ref.p.itab) == bytes(d.p.itab), name
        assert list(ref.arg_numel)[:ref.nargs] == list(d.arg_numel)[:d.nargs], name
        assert list(ref.arg_dtype)[:ref.nargs] == list(d.arg_dtype)[:d.nargs], name
