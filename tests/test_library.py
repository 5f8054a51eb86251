"""The C-ABI library on the CPU: it loads, exports every entry point include/*.h declares, the
ctypes binding covers them, and the ops refuse non-CUDA tensors (there is no CPU path)."""

import ctypes
import os
import re

import pytest
import torch

from conftest import ROOT


def _declared():
    names = set()
    inc = os.path.join(ROOT, "include")
    for f in os.listdir(inc):
        if f.endswith(".h"):
            src = open(os.path.join(inc, f)).read()
            src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
            names |= set(re.findall(r"\b(qb_[a-z0-9_]+)\s*\(", src))
    return names


def test_library_loads_and_exports_every_declared_symbol():
    from hackathon_b200 import _lib
    lib = _lib.load()
    declared = _declared()
    assert declared, "no declarations found"
    for name in sorted(declared):
        assert hasattr(lib, name), f"{name} declared in include/ but not exported"
        ctypes.cast(getattr(lib, name), ctypes.c_void_p)
    assert declared <= set(_lib.exported_symbols()), declared - set(_lib.exported_symbols())
    assert lib.qb_abi_version() >= 1


def test_error_message_plumbing_without_gpu():
    """Argument checks run before any CUDA call, so they work here."""
    from hackathon_b200 import _lib
    lib = _lib.load()
    rc = lib.qb_nf4_dequant(None, 3, None, 0, None, None, 0.0, 64, 256, None, None, 2, None)
    assert rc == 1
    assert b"even" in lib.qb_last_error()
    rc = lib.qb_rmsnorm_fwd(None, 0, 0, None, 0, None, 0, 0, None, 4, 0, 1e-6, None)
    assert rc == 1 and b"bad shape" in lib.qb_last_error()
    with pytest.raises(RuntimeError, match="qb_swiglu_fwd failed"):
        _lib.call("qb_swiglu_fwd", None, None, None, 2, -1, None)
    # two-segment GEMM: layouts other than the projection's two are refused before any launch
    fake = 1 << 20
    with pytest.raises(RuntimeError, match="K-major"):
        _lib.call("qb_gemm2_bf16", fake, 64, 1, fake, 64, 0, 64, fake, 64, 0, fake, 64, 0, 64,
                  fake, 64, 2, None, None, 0, 128, 128, None)
    with pytest.raises(RuntimeError, match="bad K"):
        _lib.call("qb_gemm2_bf16", fake, 64, 0, fake, 64, 0, 0, fake, 64, 0, fake, 64, 0, 64,
                  fake, 64, 2, None, None, 0, 128, 128, None)
    with pytest.raises(RuntimeError, match="residual row stride"):
        _lib.call("qb_gemm2_bf16", fake, 64, 0, fake, 64, 0, 64, None, 0, 0, None, 0, 0, 0,
                  fake, 128, 2, None, fake, 64, 128, 128, None)
    # the failure-path self-test refuses limits outside 1 ms .. 2 s before launching anything
    assert lib.qb_selftest_bounded_wait(10, None) == 1
    assert lib.qb_selftest_bounded_wait(10_000_000_000, None) == 1
    with pytest.raises(RuntimeError, match="mask row stride"):
        _lib.call("qb_gemm_bf16_mask_acc", fake, 64, fake, 64, 1, fake, 3, 1.0, fake, 128, 128,
                  128, 64, None)
    # mask bits drawn ahead: grid caps outside 0..8 and p >= 1 are refused before any launch
    with pytest.raises(RuntimeError, match="ctas_per_sm"):
        _lib.call("qb_dropout_bits", fake, 16, 64, 1, 0.1, 9, None)
    with pytest.raises(RuntimeError, match="p must be < 1"):
        _lib.call("qb_dropout_bits", fake, 16, 64, 1, 1.0, 2, None)
    assert lib.qb_dropout_bits(None, 0, 64, 1, 0.1, 2, None) == 0     # empty: nothing to do
    # the launch monitor's report reads host memory only: it answers without a GPU (nothing
    # launched yet) and refuses a missing buffer or an impossible device index
    buf = ctypes.create_string_buffer(256)
    assert lib.qb_monitor_report(0, buf, len(buf)) == 0
    assert b"no launch monitor" in buf.value
    assert lib.qb_monitor_report(0, None, 16) == 1
    assert lib.qb_monitor_report(99, buf, len(buf)) == 1


@pytest.mark.parametrize("op", ["rmsnorm", "rope", "swiglu", "dropout", "dequant"])
def test_ops_refuse_cpu_tensors(op):
    import hackathon_b200 as hb
    from hackathon_b200 import lora, nf4, rmsnorm, rope, swiglu
    x = torch.randn(2, 4, 8)
    with pytest.raises(RuntimeError, match="CUDA"):
        if op == "rmsnorm":
            rmsnorm.rmsnorm(x, torch.ones(8), 1e-6)
        elif op == "rope":
            rope.TritonRoPE.apply(x[None], x[None], x, x)
        elif op == "swiglu":
            swiglu.swiglu(x, x)
        elif op == "dropout":
            lora.DropoutCast.apply(x, 0.1, 1, torch.float32)
        else:
            st = nf4.QuantState(absmax=torch.ones(1), shape=(2, 4), blocksize=64)
            nf4.dequantize_nf4(torch.zeros(4, dtype=torch.uint8), st)
    assert hb.PATCHES == ("rmsnorm", "rope", "cross_entropy", "lora")


def test_quant_state_admission():
    from hackathon_b200.nf4 import QuantState, supported
    s2 = QuantState(absmax=torch.ones(1), blocksize=256, quant_type="dynamic")
    assert supported(QuantState(absmax=torch.ones(1), shape=(4, 64), blocksize=64, state2=s2))
    assert not supported(QuantState(absmax=torch.ones(1), shape=(4, 64), blocksize=63))
    assert not supported(QuantState(absmax=torch.ones(1), shape=(4, 4, 4), blocksize=64))
    assert not supported(QuantState(absmax=torch.ones(1), shape=(4, 64), blocksize=64,
                                    quant_type="fp4"))
    assert not supported(None)


def test_shift_labels_and_chunked_step_host_logic():
    from hackathon_b200.cross_entropy import ChunkedStep, shift_labels_of
    labels = torch.tensor([[1, 2, 3], [4, -100, 6]])
    assert shift_labels_of(labels).tolist() == [[2, 3, -100], [-100, 6, -100]]
    target = shift_labels_of(labels)
    pred = torch.tensor([[2, 0, 0], [0, 6, 1]])
    st = ChunkedStep(torch.zeros(2, 3), torch.zeros(2, 3), pred, target)
    assert int(st.labelled) == 3 and int(st.correct) == 2


def test_rope_supported_guard():
    from hackathon_b200.rope import _supported
    q = torch.randn(1, 2, 3, 8)
    assert not _supported(q, q, q[0], q[0], 1)   # CPU tensors go to the original


def test_apply_is_idempotent_without_gpu():
    import hackathon_b200 as hb
    from transformers.models.qwen2 import modeling_qwen2 as m
    hb.apply()
    first = m.Qwen2RMSNorm.forward
    hb.apply()
    assert m.Qwen2RMSNorm.forward is first
    # patched forward hands CPU tensors to the original implementation
    norm = m.Qwen2RMSNorm(8)
    x = torch.randn(2, 8)
    want = norm.weight * (x * torch.rsqrt(x.pow(2).mean(-1, keepdim=True) + 1e-6))
    torch.testing.assert_close(norm(x), want)


def test_library_is_built_from_the_current_sources():
    """The in-tree library is newer than every CUDA source and header it is built from, so the
    tests here and on the GPU exercise the code in the tree, not an older build left behind by a
    rebuild that failed."""
    from hackathon_b200.csrc import build as b
    assert os.path.exists(b.LIB), "library not built: python -m hackathon_b200.csrc.build"
    lib_t = os.path.getmtime(b.LIB)
    srcs = [os.path.join(b.HERE, f) for f in b._sources()] + b._headers()
    stale = [os.path.relpath(p, ROOT) for p in srcs if os.path.getmtime(p) > lib_t]
    assert not stale, f"sources newer than the library (rebuild): {stale}"


def test_ctypes_bindings_match_the_header_declarations():
    """Every binding in _lib passes exactly the arguments its C declaration takes, each of the
    same kind (pointer / int64 / int / float / uint64): a shifted or missing argument would reach
    a kernel launch as a wrong size or address."""
    from hackathon_b200 import _lib
    src = open(os.path.join(ROOT, "include", "qlora_b200.h")).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    decls = re.findall(r"\b(?:int|int64_t|const char\*)\s+(qb_[a-z0-9_]+)\s*\(([^)]*)\)\s*;", src)
    assert len(decls) >= 30

    def c_kind(p):
        p = p.strip()
        if p in ("", "void"):
            return None
        if "*" in p or p.startswith("cudaStream_t"):
            return "ptr"
        t = p.rsplit(" ", 1)[0].replace("const ", "").strip()
        return {"int64_t": "i64", "int": "i32", "float": "f32", "uint64_t": "u64"}[t]

    def py_kind(t):
        if t in (ctypes.c_void_p, ctypes.c_char_p) or isinstance(t, type) and \
                issubclass(t, ctypes._Pointer):
            return "ptr"
        return {ctypes.c_int64: "i64", ctypes.c_int: "i32", ctypes.c_float: "f32",
                ctypes.c_uint64: "u64"}[t]

    for name, params in decls:
        want = [k for k in map(c_kind, params.split(",")) if k is not None]
        have = [py_kind(t) for t in _lib._SIGNATURES[name]]
        assert have == want, f"{name}: binding {have} vs declaration {want}"


def test_mask_job_layout_and_argument_checks():
    """The ctypes qb_mask_job has the C struct's size; the gate/up GEMM with mask jobs refuses
    too many jobs, bad shapes and unaligned bits before any CUDA call."""
    import ctypes
    from hackathon_b200 import _lib
    from hackathon_b200.gemm import MaskJob
    assert _lib.load().qb_mask_job_size() == ctypes.sizeof(MaskJob) == 40
    fake = 1 << 20
    args = (fake, 896, fake, fake, 896, 896, None, 0, None, None, 0, 0, fake, 1536, None, None,
            1536, 128, 1536)

    def run(jobs, n):
        arr = (MaskJob * max(len(jobs), 1))(*jobs)
        _lib.call("qb_gemm_gateup_swiglu_masks", *args, arr, n, None)

    ok = MaskJob(fake, 16, 64, 1, 0.1)
    with pytest.raises(RuntimeError, match="mask jobs"):
        run([ok] * 9, 9)
    with pytest.raises(RuntimeError, match="bad shape"):
        run([ok, MaskJob(fake, 16, 0, 1, 0.1)], 2)
    with pytest.raises(RuntimeError, match="p must be < 1"):
        run([MaskJob(fake, 16, 64, 1, 1.0)], 1)
    with pytest.raises(RuntimeError, match="4-byte aligned"):
        run([MaskJob(fake + 2, 16, 64, 1, 0.1)], 1)


def test_dropout_apply_multi_argument_checks():
    """qb_dropout_apply_multi refuses 0 or more than 4 outputs, an empty output table and
    columns that are not a multiple of 8 before any CUDA call."""
    import ctypes
    from hackathon_b200 import _lib
    fake = 1 << 20
    bits = (ctypes.c_void_p * 5)(*([fake] * 5))
    outs = (ctypes.c_void_p * 5)(*([fake] * 5))
    lds = (ctypes.c_int64 * 5)(*([64] * 5))
    scs = (ctypes.c_float * 5)(*([2.0] * 5))
    for n in (0, 5):
        with pytest.raises(RuntimeError, match="1..4 outputs"):
            _lib.call("qb_dropout_apply_multi", fake, 2, 64, n, bits, outs, 2, lds, scs, 16, 64,
                      None)
    with pytest.raises(RuntimeError, match="null output table"):
        _lib.call("qb_dropout_apply_multi", fake, 2, 64, 2, None, outs, 2, lds, scs, 16, 64, None)
    with pytest.raises(RuntimeError, match="multiple of 8"):
        _lib.call("qb_dropout_apply_multi", fake, 2, 64, 2, bits, outs, 2, lds, scs, 16, 60, None)


def test_pack_segment_layout_and_table():
    """The Python table of qb_adapter_pack has the C struct's size, and its chunk offsets are the
    running sum of each segment's 2048-element chunks (host only: no launch)."""
    import numpy as np
    import torch
    from hackathon_b200 import _lib
    from hackathon_b200.lora import PACK_CHUNK, PACK_SEGMENT, pack_table
    assert _lib.load().qb_pack_segment_size() == np.dtype(PACK_SEGMENT).itemsize == 56
    src = [torch.zeros(64, 3584), torch.zeros(512, 64), torch.zeros(0, 64), torch.zeros(3, 5)]
    dst = [torch.zeros(s.shape, dtype=torch.bfloat16) for s in src]
    raw, chunks = pack_table([(s, d, 2.0) for s, d in zip(src, dst)])
    table = np.frombuffer(raw, dtype=np.dtype(PACK_SEGMENT))
    want = np.cumsum([0] + [(s.numel() + PACK_CHUNK - 1) // PACK_CHUNK for s in src])
    assert list(table["first_chunk"]) == list(want[:-1]) and chunks == want[-1]
    assert list(table["rows"]) == [64, 512, 0, 3] and list(table["src_ld"]) == [3584, 64, 64, 5]
    assert table["src"][0] == src[0].data_ptr() and table["dst"][3] == dst[3].data_ptr()
    with pytest.raises(TypeError):
        pack_table([(src[0].double(), dst[0], 1.0)])
    with pytest.raises(ValueError):
        pack_table([(src[0], dst[1], 1.0)])


def test_mask_and_product_bookkeeping_on_the_host():
    """The host logic that decides which dropout masks a gate/up GEMM draws, which recorded masks
    a projection may use, and when a rank-r product is kept for the recompute (no launch)."""
    import torch
    from hackathon_b200 import qlora

    class Proj:
        def __init__(self, in_features, p=0.05, fused=True, training=True):
            self.in_features, self.p, self.fused, self.training = in_features, p, fused, training
            self.quant_state = None

    a, b, off, odd = Proj(3584), Proj(18944), Proj(3584, p=0.0), Proj(3580)
    qlora.MASKS.clear()
    try:
        qlora.MASKS[(id(b), 7)] = torch.zeros((16, 592), dtype=torch.int32)   # drawn already
        jobs = qlora.gemm_mask_jobs([(a, 5), (b, 7), (off, 9), (odd, 11)], 16, "cpu")
        assert [(j[1], j[2], j[3], j[4]) for j in jobs] == [(16, 3584, 5, 0.05)]
        assert jobs[0][0].shape == (16, 112) and jobs[0][0].dtype == torch.int32
        assert qlora.MASKS[(id(a), 5)] is jobs[0][0]
        bits, scale = qlora.recorded_mask(a, 5, 16)
        assert bits is jobs[0][0] and abs(scale - 1 / 0.95) < 1e-12
        assert qlora.recorded_mask(a, 5, 32) is None          # other rows
        assert qlora.recorded_mask(off, 9, 16) is None        # no dropout
        assert qlora.recorded_mask(Proj(3584, training=False), 5, 16) is None
        # on the CPU no projection takes the fused path: every shared dropout is left to it
        x = torch.zeros(16, 3584, dtype=torch.bfloat16)
        assert qlora.shared_dropouts(x, [(a, 5), (a, 5)]) == [None, None]
    finally:
        qlora.MASKS.clear()
    assert qlora._keep_uprod(False, True) and not qlora._keep_uprod(True, True)
    assert not qlora._keep_uprod(False, False)
