"""CPU checks of the native boundary: libokc_b200.so loads without a GPU, exports every
symbol that include/okc_b200.h declares, and its argument validation rejects bad calls
before touching the device."""

import re
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent


def declared_functions():
    src = (ROOT / "include" / "okc_b200.h").read_text()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return sorted(set(re.findall(r"\b(okc_[a-z0-9_]+)\s*\(", src)))


@pytest.fixture(scope="module")
def lib():
    from okc_b200 import _lib
    return _lib.load()


def test_every_declared_symbol_is_exported(lib):
    names = declared_functions()
    assert len(names) >= 12
    for n in names:
        assert hasattr(lib, n), n


def test_ctypes_signatures_cover_header():
    from okc_b200 import _lib
    assert sorted(_lib.SIGNATURES) == declared_functions()


def test_version(lib):
    assert lib.okc_version().decode().startswith("okc_b200")


def test_validation_without_device(lib):
    from okc_b200 import _lib
    # null pointers / bad shapes are rejected before any CUDA call
    assert lib.okc_gemm_bf16(None, 0, None, 0, None, 0, None, 1, 1, 1, 0, None, 0, None) == _lib.OKC_ERR_INVALID
    assert lib.okc_gemm_bf16(8, 8, 16, 8, 32, 8, None, 1, 8, 12, 0, None, 0, None) == _lib.OKC_ERR_INVALID  # K % 8
    assert lib.okc_gemm_bf16(8, 8, 16, 8, 32, 8, None, 1, 8, 8, 0, None, 0, None) == _lib.OKC_ERR_ALIGNMENT
    assert lib.okc_gemm_bf16(16, 8, 16, 8, 33, 8, None, 1, 8, 8, 0, None, 0, None) == _lib.OKC_ERR_ALIGNMENT
    assert lib.okc_attn_decode_fp8(16, 64, 16, 16, 16, 4, 16, 16, 16, 16, 64, 1, 9, 8, 64, 16, 4, 0.1, 1,
                                   None, 0, None) == _lib.OKC_ERR_INVALID  # Hq % Hkv
    assert lib.okc_attn_decode_fp8(16, 64, 16, 16, 16, 4, 16, 16, 16, 16, 64, 1, 8, 8, 96, 16, 4, 0.1, 1,
                                   None, 0, None) == _lib.OKC_ERR_INVALID  # D = 96
    assert lib.okc_moe_route(16, 16, 16, 16, None, 1, 100, 64, 8, 1, None) == _lib.OKC_ERR_INVALID  # H % 256
    assert lib.okc_moe_permute(16, 20000, 8, 0, 64, 8, 16, 16, 16, 16, 100, None) == _lib.OKC_ERR_INVALID
    # residual boundary: H > 16384, ld_branch < H, a misaligned pointer
    assert lib.okc_residual_boundary(16, 16, 16392, 16, 16, None, 16, 16, 16, None, 1, 16392, 1e-8, 1e-5,
                                     None) == _lib.OKC_ERR_INVALID
    assert lib.okc_residual_boundary(16, 16, 4088, 16, 16, None, 16, 16, 16, None, 1, 4096, 1e-8, 1e-5,
                                     None) == _lib.OKC_ERR_INVALID
    assert lib.okc_residual_boundary(16, 16, 4096, 16, 16, 24, 16, 16, 16, None, 1, 4096, 1e-8, 1e-5,
                                     None) == _lib.OKC_ERR_ALIGNMENT
    # post-expert norm: H above the combine's 8192
    assert lib.okc_moe_experts_w4a16_post(*([16] * 13), 4, 8, 16384, 1536, 0, 32, 0, 16, 1e-8, 16, 1 << 30,
                                          None) == _lib.OKC_ERR_INVALID


def test_workspace_queries(lib):
    from okc_b200 import _lib
    n = lib.okc_attn_decode_workspace_bytes(64, 64, 8, 128, 148)
    rows = (148 + 64) * 1 * 64
    assert n == (256 + ((rows * 8 + 255) // 256) * 256 + ((rows * 128 * 4 + 255) // 256) * 256
                 + ((64 + 1) * 4 + 255) // 256 * 256   # + the unit prefix for the merge
                 + (64 * 8 * (2048 + 32) + 255) // 256 * 256)  # + two-term e4m3 queries and scales
    assert lib.okc_attn_decode_workspace_bytes(8, 8, 1, 128, 10) > lib.okc_attn_decode_workspace_bytes(8, 8, 8, 128, 10)
    assert lib.okc_moe_experts_workspace_bytes(256, 8, 4096, 1536) > 256


def _header_prototypes():
    src = (ROOT / "include" / "okc_b200.h").read_text()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    src = re.sub(r"//[^\n]*", "", src)
    src = re.sub(r"#[^\n]*", "", src)
    protos = {}
    for ret, name, params in re.findall(r"([A-Za-z_][\w \t\*]*?)\s*\b(okc_[a-z0-9_]+)\s*\(([^)]*)\)\s*;", src):
        ps = [p.strip() for p in params.split(",") if p.strip() and p.strip() != "void"]
        protos[name] = (ret.strip(), ps)
    return protos


def _kind_of_c(decl: str) -> str:
    decl = " ".join(decl.split())
    if "*" in decl or decl.startswith("okc_stream_t"):
        return "ptr"
    base = decl.replace("const ", "").rsplit(" ", 1)[0] if " " in decl.replace("const ", "") else decl
    base = base.strip()
    return {"int": "i32", "long long": "i64", "int64_t": "i64", "size_t": "size", "float": "f32",
            "double": "f64"}.get(base, "?" + base)


def _kind_of_ctypes(t) -> str:
    import ctypes as C
    if t in (C.c_void_p, C.c_char_p) or (isinstance(t, type) and issubclass(t, C._Pointer)):
        return "ptr"
    if t is C.c_size_t:
        return "size"
    if t in (C.c_int, C.c_int32):
        return "i32"
    if t in (C.c_longlong, C.c_int64):
        return "i64"
    if t is C.c_float:
        return "f32"
    if t is C.c_double:
        return "f64"
    return "?" + repr(t)


def test_ctypes_signatures_match_header_prototypes():
    """Every ctypes argtype / restype has the kind (pointer, int, 64-bit int, size_t, float)
    of the header's parameter in the same position: a mismatch would pass arguments wrongly."""
    from okc_b200 import _lib
    protos = _header_prototypes()
    assert sorted(protos) == declared_functions()
    bad = []
    for name, (ret, params) in protos.items():
        restype, argtypes = _lib.SIGNATURES[name]
        want = [_kind_of_c(p) for p in params]
        got = [_kind_of_ctypes(t) for t in argtypes]
        if want != got:
            bad.append(f"{name}: header {want} vs ctypes {got}")
        rk = "ptr" if "*" in ret else _kind_of_c(ret + " r")
        if rk != _kind_of_ctypes(restype):
            bad.append(f"{name}: returns {ret} vs ctypes {restype}")
    assert not bad, "\n".join(bad)


def _kernel_bodies(pattern=r"__global__\s+void\s+(?:__launch_bounds__\([^)]*\)\s*)?(\w+)\s*\("):
    bodies = {}
    for f in sorted((ROOT / "okc_b200" / "csrc").glob("*.cu")):
        src = f.read_text()
        for m in re.finditer(pattern, src):
            i = src.index("{", m.end())
            depth, j = 0, i
            while True:
                if src[j] == "{":
                    depth += 1
                elif src[j] == "}":
                    depth -= 1
                    if depth == 0:
                        break
                j += 1
            bodies[m.group(1)] = src[i:j]
    return bodies


def test_every_pdl_launched_kernel_waits_before_returning():
    """Kernels launched with programmatic dependent launch (okc_host::launch_k) may start before
    their predecessor finished, so each must execute griddepcontrol.wait (pdl_wait) before it
    returns or reads the predecessor's output; then a kernel's completion implies every earlier
    kernel's, which the cross-GPU protocols rely on.  Kernels launched with <<<>>> are stream
    ordered and exempt."""
    src = "".join(f.read_text() for f in (ROOT / "okc_b200" / "csrc").glob("*.cu"))
    launched = set(re.findall(r"launch_k\(\s*(?:okc::)?(\w+)", src))
    bodies = _kernel_bodies()
    # device functions a kernel delegates to (a kernel body that is a call of a templated body
    # function): their text is spliced in place of the call, one level deep
    helpers = _kernel_bodies(r"__device__\s+(?:__forceinline__\s+|__noinline__\s+)?void\s+(\w+)\s*\(")
    assert launched, "no launch_k call found"
    bad = []
    for name in sorted(launched):
        assert name in bodies, f"launch_k of unknown kernel {name}"
        body = bodies[name]
        for h, hb in helpers.items():
            body = re.sub(r"\b" + h + r"\s*(<[^;{}]*>)?\s*\([^;]*\);", lambda _m, hb=hb: hb, body)
        w = body.find("pdl_wait()")
        if w < 0:
            bad.append(f"{name}: no pdl_wait")
            continue
        early = [r.start() for r in re.finditer(r"\breturn\b", body) if r.start() < w]
        if early:
            bad.append(f"{name}: returns before pdl_wait")
        # a warp-specialised kernel splits into roles with an if / else-if chain on the warp
        # index; the wait must come before that split, so that every role has executed it
        split = re.search(r"\}\s*else\s+if\s*\(\s*warp\b", body)
        if split and split.start() < w:
            bad.append(f"{name}: role split before pdl_wait")
    assert not bad, bad


def test_every_device_spin_wait_is_bounded():
    """Device code polls in exactly two places, both bounded by kWaitNs of %globaltimer:
    mbar_wait (common.cuh: mbarrier phases) and wait_flag (tp_comm.cu: cross-GPU flags).  No
    other code issues mbarrier.try_wait / test_wait, loops on an acquire or volatile load in a
    while condition, or polls one inside an unconditional loop (for (;;), while (true),
    do { } while)."""
    csrc = ROOT / "okc_b200" / "csrc"
    files = {f.name: f.read_text() for f in list(csrc.glob("*.cu")) + list(csrc.glob("*.cuh"))}
    for name, src in files.items():
        code = re.sub(r"//[^\n]*", "", src)
        if name != "common.cuh":
            assert "mbarrier.try_wait" not in code and "mbarrier.test_wait" not in code, name
            assert "mbar_try_wait(" not in code, f"{name}: polls an mbarrier outside mbar_wait"
        for m in re.finditer(r"while\s*\(([^)]*(?:\([^)]*\)[^)]*)*)\)", code):
            cond = m.group(1)
            if "ld_acquire" in cond or "volatile" in cond or "ld.acquire" in cond:
                head = code[:m.start()]
                fn = re.findall(r"__device__[^{;]*?\b(\w+)\s*\([^;{]*\)\s*\{", head)
                assert fn and fn[-1] == "wait_flag", f"{name}: flag polling outside wait_flag"
        # unconditional loops (for (;;), while (true/1), do { } while) that poll a flag
        for m in re.finditer(r"for\s*\(\s*;\s*;\s*\)|while\s*\(\s*(?:true|1)\s*\)|\bdo\s*\{", code):
            start = code.index("{", m.start())
            depth, i = 0, start
            while i < len(code):
                depth += code[i] == "{"
                depth -= code[i] == "}"
                if depth == 0:
                    break
                i += 1
            loop = code[start:i]
            if any(k in loop for k in ("ld_acquire", "ld.acquire", "volatile", "mbar_try_wait", "try_wait")):
                head = code[:m.start()]
                fn = re.findall(r"__device__[^{;]*?\b(\w+)\s*\([^;{]*\)\s*\{", head)
                assert fn and fn[-1] in ("wait_flag", "mbar_wait"), f"{name}: unbounded-looking poll loop"
    common = re.sub(r"//[^\n]*", "", files["common.cuh"])
    body = common[common.index("bool mbar_wait("):]
    body = body[:body.index("\n}\n")]
    assert "kWaitNs" in body and "globaltimer" in body
    tp = re.sub(r"//[^\n]*", "", files["tp_comm.cu"])
    body = tp[tp.index("bool wait_flag("):]
    body = body[:body.index("\n}\n")]
    assert "kWaitNs" in body and "globaltimer" in body
