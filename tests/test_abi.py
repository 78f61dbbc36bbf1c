"""The C-ABI library: loads, exports every symbol include/attn_rt.h declares,
and rejects bad operands with the reference verifier's rules (no GPU needed:
validation happens before any device call)."""
import ctypes
import os
import re
import subprocess

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "attn_rt.h")


def declared_functions():
    text = open(HEADER).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    text = "\n".join(ln for ln in text.splitlines() if not ln.lstrip().startswith("#"))
    return sorted(set(re.findall(r"\b(\w+)\s*\([^;{]*\)\s*;", text)) - {"sizeof"})


def test_header_declares_the_entry_points():
    names = declared_functions()
    assert "attn_fwd" in names and "_mlir_ciface_attn_fused_f32_mask" in names
    assert len(names) >= 16


def test_library_exports_every_declared_symbol(pkg):
    pkg.lib()
    out = subprocess.run(["nm", "-D", "--defined-only", pkg.LIB_PATH], capture_output=True,
                         text=True, check=True).stdout
    exported = {ln.split()[-1] for ln in out.splitlines() if ln.strip()}
    missing = [n for n in declared_functions() if n not in exported]
    assert not missing, missing


def test_version_and_status_strings(pkg):
    L = pkg.lib()
    assert L.attn_rt_version() >> 16 == 1
    for code, text in pkg.STATUS.items():
        assert L.attn_rt_status_string(code).decode() == text


def _desc(pkg, **kw):
    d = pkg.AttnDesc()
    d.dtype, d.out_dtype, d.mask_kind = pkg.ATTN_BF16, pkg.ATTN_BF16, pkg.MASK_CAUSAL
    d.B, d.Hq, d.Hkv, d.Nq, d.Nk, d.D = 1, 4, 2, 256, 256, 128
    for s in (d.q_stride, d.o_stride):
        s[0], s[1], s[2] = 4 * 256 * 128, 256 * 128, 128
    for s in (d.k_stride, d.v_stride):
        s[0], s[1], s[2] = 2 * 256 * 128, 256 * 128, 128
    d.q = d.k = d.v = d.o = 0x10000
    d.scale = 0.125
    d.q_descale = d.k_descale = d.v_descale = 1.0
    for k, v in kw.items():
        setattr(d, k, v)
    return d


@pytest.mark.parametrize("field,value,code", [
    ("Hkv", 3, -2),          # heads not a multiple
    ("Nk", -1, -2),          # negative extent
    ("D", 96, -8),           # bf16 head_dim not built
    ("dtype", 7, -4),
    ("mask_kind", 2, -1),    # dense without a mask pointer
    ("q", 0x10008, -5),      # misaligned
    ("flags", 1, -1),
    ("k_descale_blocks", 0x20000, -4),  # per-block descales need e4m3 inputs
])
def test_validation_codes(pkg, field, value, code):
    L = pkg.lib()
    d = _desc(pkg, **{field: value})
    assert L.attn_fwd(ctypes.byref(d), None) == code
    assert pkg.last_error()


def test_block_descale_alignment(pkg):
    """e4m3 with a misaligned per-block descale array is rejected before launch."""
    d = _desc(pkg, dtype=pkg.ATTN_E4M3, q_descale_blocks=0x20002)
    assert pkg.lib().attn_fwd(ctypes.byref(d), None) == -5
    assert "4-byte" in pkg.last_error()


def test_null_descriptor(pkg):
    assert pkg.lib().attn_fwd(None, None) == -1


def test_no_device_is_reported_not_faked(pkg):
    """On a machine without an sm_100 GPU a valid call fails loudly."""
    torch = pytest.importorskip("torch")
    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    d = _desc(pkg)
    assert pkg.lib().attn_fwd(ctypes.byref(d), None) == -9


def test_device_memory_helpers_without_a_gpu(pkg):
    """attn_rt_alloc / free / copy check their arguments before any device
    call, and report a missing GPU instead of faking memory."""
    torch = pytest.importorskip("torch")
    L = pkg.lib()
    p = ctypes.c_void_p()
    assert L.attn_rt_alloc(None, 16) == -1
    assert L.attn_rt_alloc(ctypes.byref(p), 0) == -1
    assert L.attn_rt_free(None) == 0
    assert L.attn_rt_copy(None, None, 0, None) == 0
    assert L.attn_rt_copy(None, ctypes.byref(p), 8, None) == -1
    if not torch.cuda.is_available():
        assert L.attn_rt_alloc(ctypes.byref(p), 256) == -9


def _pass_callees():
    """(callee, argument count) for every call the --attention-to-runtime
    pass can emit, following its rules (mlir/RuntimeLoweringPass.cpp): f32
    lowers in rank 2 or 4, the other types in rank 4; a general i1 mask only
    for rank-2 f32 and rank-4 bf16; arguments Q, K, V, scale, three descales
    for e4m3, the mask, O, and an LSE memref for the non-f32 entries."""
    src = open(os.path.join(ROOT, "mlir-flashattention_b200", "mlir",
                            "RuntimeLoweringPass.cpp")).read()
    assert 'std::string callee = ("attn_fused_" + dt + "_").str();' in src
    assert '(dt == "f32" && rank == 2) || (dt == "bf16" && rank == 4)' in src
    assert '(rank == 4 && maskRank == 2) ? "mask2d"' in src
    assert "cf::AssertOp" in src  # the returned status is checked
    out = []
    for dt in ("f32", "bf16", "f16", "e4m3"):
        for rank in (2, 4):
            if dt != "f32" and rank != 4:
                continue
            for kind in ("nomask", "causal", "mask", "mask2d"):
                if kind == "mask" and not ((dt == "f32" and rank == 2) or (dt == "bf16" and rank == 4)):
                    continue
                if kind == "mask2d" and not (dt == "bf16" and rank == 4):
                    continue  # a rank-2 mask on rank-4 bf16 operands
                name = f"attn_fused_{dt}_{kind}" + ("_4d" if rank == 4 else "")
                nargs = 4 + (3 if dt == "e4m3" else 0) + (1 if kind.startswith("mask") else 0) + \
                    1 + (1 if dt != "f32" else 0)
                out.append((name, nargs))
    return out


def test_every_call_the_lowering_pass_emits_is_declared_with_its_arity():
    text = re.sub(r"/\*.*?\*/", "", open(HEADER).read(), flags=re.S)
    protos = {m.group(1): m.group(2) for m in
              re.finditer(r"_mlir_ciface_(\w+)\s*\(([^;{]*)\)\s*;", text)}
    callees = _pass_callees()
    assert len(callees) == 13
    for name, nargs in callees:
        assert name in protos, name
        assert protos[name].count(",") + 1 == nargs, (name, protos[name])


def test_every_call_the_lowering_pass_emits_is_exported(pkg):
    pkg.lib()
    out = subprocess.run(["nm", "-D", "--defined-only", pkg.LIB_PATH], capture_output=True,
                         text=True, check=True).stdout
    exported = {ln.split()[-1] for ln in out.splitlines() if ln.strip()}
    missing = ["_mlir_ciface_" + n for n, _ in _pass_callees() if "_mlir_ciface_" + n not in exported]
    assert not missing, missing
