"""The Rust integration crate (crates/vocal-retrieval-b200) against the
library it binds, without a Rust toolchain: every function its `extern "C"`
blocks declare from libvfr_retrieval.so is exported by the built library,
every entry point include/vfr_retrieval.h declares has a Rust binding, the
`#[repr(C)]` structs list the header's fields in the header's order, and the
reference's three retrieval names keep the reference's argument count
(crates/vocal-tensorrt/src/ffi.rs:174-199: 14, 1 and 7 arguments)."""
import ctypes
import os
import re

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
CRATE = os.path.join(ROOT, "crates", "vocal-retrieval-b200")
FFI = os.path.join(CRATE, "src", "ffi.rs")
HEADER = os.path.join(ROOT, "include", "vfr_retrieval.h")


def _extern_fns():
    """{name: argument count} of the library functions in ffi.rs's extern
    blocks (the CUDA runtime block, functions named cuda*, is not ours)."""
    text = open(FFI).read()
    out = {}
    for block in re.findall(r'unsafe extern "C" \{(.*?)\n\}', text, re.S):
        for name, args in re.findall(r"pub fn ([a-z_][a-z0-9_]*)\((.*?)\)\s*(?:->[^;]*)?;", block, re.S):
            if name.startswith("cuda"):
                continue
            out[name] = len([a for a in args.split(",") if a.strip()])
    return out


def _header_struct(name):
    text = open(HEADER).read()
    body = re.search(r"typedef struct %s \{(.*?)\} %s;" % (name, name), text, re.S).group(1)
    return re.findall(r"([a-z_][a-z0-9_]*)(?:\[\d+\])?;", re.sub(r"/\*.*?\*/", "", body, flags=re.S))


def _rust_struct(name):
    text = open(FFI).read()
    body = re.search(r"pub struct %s \{(.*?)\n\}" % name, text, re.S).group(1)
    return re.findall(r"pub ([a-z_][a-z0-9_]*):", body)


def test_every_rust_extern_is_exported(native):
    fns = _extern_fns()
    assert len(fns) >= 40
    missing = [n for n in fns if not hasattr(native, n)]
    assert not missing, missing


def test_every_header_entry_point_has_a_binding():
    from vfr import lib

    declared = set(lib.declared_symbols())
    assert declared, "no declarations parsed from the header"
    assert declared <= set(_extern_fns()), sorted(declared - set(_extern_fns()))


def test_reference_names_keep_their_arity():
    fns = _extern_fns()
    assert fns["vocal_faiss_gpu_create"] == 14
    assert fns["vocal_faiss_gpu_destroy"] == 1
    assert fns["vocal_faiss_gpu_blend"] == 7
    assert fns["vocal_retrieval_protect"] == 10


def test_repr_c_structs_match_the_header():
    assert _rust_struct("VfrOptions") == _header_struct("VfrOptions")
    assert _rust_struct("VfrIpcRows") == _header_struct("VfrIpcRows")
    assert _rust_struct("Stream") == ["stream"]


def test_struct_sizes_match_the_python_mirror():
    """The ctypes mirrors (vfr/lib.py) of the same structs have the C sizes
    the Rust #[repr(C)] definitions produce (same field types in order)."""
    from vfr import lib

    assert ctypes.sizeof(lib.Options) == 4 * 4 + 8 * 2
    assert ctypes.sizeof(lib.IpcRows) == 64 + 64 + 8 + 8 + 4 * 4
