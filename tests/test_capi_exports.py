"""The C-ABI library builds, loads, and exports every symbol the header
declares (no compute calls: this runs without a GPU)."""
import ctypes as C
import os
import re

import pytest

from marian_cuda import _lib as L
from marian_cuda import build

HEADER = os.path.join(build.REPO, "include", "marian_cuda.h")


def declared():
    text = open(HEADER).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(mc_[a-z0-9_]+)\s*\(", text)))


def test_header_declares_the_expected_surface():
    names = declared()
    assert set(names) == set(L.EXPORTS), (names, L.EXPORTS)


def test_library_exports_every_declared_symbol():
    lib = C.CDLL(L.load().__dict__.get("_name", build.LIB))
    for name in declared():
        assert hasattr(lib, name), name


def test_library_is_built_for_sm100a():
    # The shared object embeds an sm_100a cubin; the build flags say so.
    assert "arch=compute_100a,code=sm_100a" in " ".join(build.ARCH)
    assert os.path.getsize(build.LIB) > 100_000


def test_engine_creation_fails_loudly_without_a_device():
    torch = pytest.importorskip("torch")
    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    lib = L.load()
    cfg = L.Config()
    lib.mc_config_default(C.byref(cfg))
    h = C.c_void_p()
    assert lib.mc_create(C.byref(cfg), C.byref(h)) == L.MC_CUDA
    assert not h.value


def test_config_validation_rejects_bad_values():
    lib = L.load()
    cfg = L.Config()
    lib.mc_config_default(C.byref(cfg))
    assert (cfg.max_inflight, cfg.page_tokens, cfg.max_length_factor, cfg.lanes) == (1024, 16, 3, 1)
    h = C.c_void_p()
    for field, bad in (("max_length_factor", 9), ("page_tokens", 12), ("lanes", 9), ("max_inflight", 0)):
        c2 = L.Config()
        lib.mc_config_default(C.byref(c2))
        setattr(c2, field, bad)
        assert lib.mc_create(C.byref(c2), C.byref(h)) == L.MC_INVALID_INPUT, field
        assert not h.value


def test_rust_binding_declares_every_header_symbol():
    # The Rust crate's raw declarations (crates/marian-cuda/src/ffi.rs) cover
    # the whole C ABI, and nothing the header lacks.
    ffi = os.path.join(build.ROOT, "crates", "marian-cuda", "src", "ffi.rs")
    text = open(ffi).read()
    rust = sorted(set(re.findall(r"pub fn (mc_[a-z0-9_]+)\s*\(", text)))
    assert rust == declared()
    # struct layouts: every mc_* struct field of the header appears in the mirror
    header = re.sub(r"/\*.*?\*/", "", open(HEADER).read(), flags=re.S)
    for name in ("mc_config", "mc_model_info", "mc_model_report", "mc_text_segment"):
        body = re.search(r"typedef struct \{([^{}]*)\}\s*" + name + ";", header).group(1)
        fields = re.findall(r"(\w+)\s*(?:,|;)", body)
        block = re.search(r"pub struct " + name + r" \{(.*?)\}", text, re.S).group(1)
        assert re.findall(r"pub (\w+):", block) == fields, name
