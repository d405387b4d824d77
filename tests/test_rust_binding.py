"""The Rust binding (small-lm-rs_b200/rust: slmkv-sys raw FFI, slmkv safe API)
against the C ABI it binds, include/slmkv.h.

The image has no Rust toolchain, so the crates cannot be compiled here; this
test holds them to the header textually: every C function is declared in
slmkv-sys with the same name, argument count and argument types (mapped
C -> Rust), the #[repr(C)] structs have the header structs' fields in order
with the same types, the status and element-type constants have the header's
values, and the safe crate calls only declared functions. With cargo on
PATH the workspace is also built."""

import re
import shutil
import subprocess
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
HEADER = ROOT / "include" / "slmkv.h"
RUST = ROOT / "small-lm-rs_b200" / "rust"
SYS = RUST / "slmkv-sys" / "src" / "lib.rs"
SAFE = RUST / "slmkv" / "src" / "lib.rs"

C_TO_RUST = {
    "int32_t": "i32", "int64_t": "i64", "uint64_t": "u64", "float": "f32",
    "const float*": "*const f32", "float*": "*mut f32",
    "const int32_t*": "*const i32", "int32_t*": "*mut i32",
    "const uint32_t*": "*const u32", "int64_t*": "*mut i64",
    "slm_ctx*": "*mut SlmCtx", "const slm_ctx*": "*const SlmCtx", "slm_ctx**": "*mut *mut SlmCtx",
    "slm_batch*": "*mut SlmBatch", "slm_batch**": "*mut *mut SlmBatch",
    "slm_sched*": "*mut SlmSched", "const slm_sched*": "*const SlmSched",
    "slm_sched**": "*mut *mut SlmSched",
    "slm_model*": "*mut SlmModel", "slm_model**": "*mut *mut SlmModel",
    "slm_stream": "*mut c_void", "const char*": "*const c_char",
    "const float* const*": "*const *const f32",
    "const slm_config*": "*const SlmConfig", "slm_config*": "*mut SlmConfig",
    "const slm_model_config*": "*const SlmModelConfig",
    "const slm_sched_config*": "*const SlmSchedConfig",
    "slm_status": "i32",
    "const slm_layer_io*": "*const SlmLayerIo",
}


def _strip_c_comments(text):
    return re.sub(r"/\*.*?\*/", "", text, flags=re.S)


def header_functions():
    src = _strip_c_comments(HEADER.read_text())
    out = {}
    for ret, name, args in re.findall(r"\n((?:const )?\w+\*?)\s+(slm_\w+)\s*\(([^;]*?)\)\s*;", src,
                                      flags=re.S):
        types = []
        for a in [x for x in (" ".join(args.split())).split(",") if x.strip()]:
            t = re.match(r"(.*?)\w+$", a.strip()).group(1)
            t = re.sub(r"\s*\*", "*", t.strip())
            if t == "const float* const*" or ("const*" in t and "float" in t):
                t = "const float* const*"
            types.append(C_TO_RUST[t])
        out[name] = (C_TO_RUST[ret.strip()] if ret.strip() != "const char*" else "*const c_char",
                     types)
    return out


def rust_functions():
    src = SYS.read_text()
    block = src[src.index('extern "C" {'):]
    out = {}
    for name, args, ret in re.findall(r"pub fn (slm_\w+)\((.*?)\)\s*->\s*([^;]+);", block, flags=re.S):
        types = [a.split(":", 1)[1].strip() for a in args.split(",") if a.strip()]
        out[name] = (ret.strip(), types)
    return out


def test_every_header_function_is_declared_with_its_types():
    hdr, rs = header_functions(), rust_functions()
    assert len(hdr) >= 49
    assert set(hdr) == set(rs), (set(hdr) ^ set(rs))
    for name, (ret, types) in hdr.items():
        assert rs[name] == (ret, types), name


def _c_struct(name):
    src = _strip_c_comments(HEADER.read_text())
    body = re.search(r"typedef struct (?:\w+ )?\{([^{}]*)\}\s*" + name + r";", src).group(1)
    return [(C_TO_RUST[t], n) for t, n in re.findall(r"(\w+)\s+(\w+);", body)]


def _rust_struct(name):
    src = SYS.read_text()
    body = re.search(r"pub struct " + name + r" \{(.*?)\}", src, flags=re.S).group(1)
    return [(t, n) for n, t in re.findall(r"pub (\w+): (\w+),", body)]


@pytest.mark.parametrize("c_name,rust_name", [("slm_config", "SlmConfig"),
                                              ("slm_model_config", "SlmModelConfig"),
                                              ("slm_sched_config", "SlmSchedConfig")])
def test_repr_c_structs_match_the_header(c_name, rust_name):
    assert _c_struct(c_name) == _rust_struct(rust_name)
    assert "#[repr(C)]" in SYS.read_text().split(f"pub struct {rust_name}")[0][-120:]


def test_layer_io_struct_matches_the_header():
    src = _strip_c_comments(HEADER.read_text())
    body = re.search(r"typedef struct slm_layer_io \{([^{}]*)\}\s*slm_layer_io;", src).group(1)
    c_fields = [(C_TO_RUST[re.sub(r"\s*\*", "*", t.strip())], n)
                for t, n in re.findall(r"([\w ]+\*)\s*(\w+);", body)]
    rs = SYS.read_text()
    rs_body = re.search(r"pub struct SlmLayerIo \{(.*?)\}", rs, flags=re.S).group(1)
    rs_fields = [(t.strip(), n) for n, t in re.findall(r"pub (\w+): ([^,]+),", rs_body)]
    assert c_fields == rs_fields
    assert "#[repr(C)]" in rs.split("pub struct SlmLayerIo")[0][-120:]


def test_constants_match_the_header():
    src = _strip_c_comments(HEADER.read_text())
    consts = dict((n, int(v)) for n, v in re.findall(r"(SLM_\w+)\s*=\s*(-?\d+)", src))
    rs = dict((n, int(v)) for n, v in re.findall(r"pub const (SLM_\w+): i32 = (-?\d+);",
                                                 SYS.read_text()))
    assert consts == rs


def test_safe_crate_calls_only_declared_functions():
    called = set(re.findall(r"sys::(slm_\w+)\(", SAFE.read_text()))
    declared = set(rust_functions())
    assert called and called <= declared, called - declared
    # the reference's KvCache methods each have a counterpart
    for method in ("layer_sequence_length", "sequence_length", "is_empty", "is_synchronized",
                   "remaining_capacity", "truncate_all", "truncate_layer", "clear",
                   "append_layer", "attend_cached_query"):
        assert f"pub fn {method}(" in SAFE.read_text(), method


@pytest.mark.skipif(shutil.which("cargo") is None, reason="no Rust toolchain in this image")
def test_workspace_builds():
    subprocess.run(["cargo", "build", "--release"], cwd=RUST, check=True)
