"""libsam3cuda loads and exports every entry point include/sam3cuda.h declares
(CPU only: no compute calls, only host-side argument validation)."""
import ctypes as C
import os
import re
import subprocess

import pytest

from conftest import PKG, ROOT

HEADER = os.path.join(ROOT, "include", "sam3cuda.h")
LIB = os.path.join(PKG, "libsam3cuda.so")


def declared_functions():
    src = open(HEADER).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    names = re.findall(r"^\s*[A-Za-z_][\w\s\*]*?\b(sam3_\w+)\s*\(", src, flags=re.M)
    return sorted(set(names))


def test_header_parses_to_entry_points():
    names = declared_functions()
    assert "sam3_linear_palette" in names and "sam3_encoder_forward_host" in names
    assert len(names) >= 28


def test_library_exports_every_declared_symbol():
    lib = C.CDLL(LIB)
    missing = [n for n in declared_functions() if not hasattr(lib, n)]
    assert not missing, missing
    out = subprocess.run(["nm", "-D", "--defined-only", LIB], capture_output=True, text=True).stdout
    exported = set(re.findall(r"\bT (sam3_\w+)", out))
    assert set(declared_functions()) <= exported


def test_binding_covers_header(sam3):
    assert set(declared_functions()) == set(sam3.SIGNATURES)


def test_struct_layouts(sam3):
    # sizes as laid out by the C compiler for the header's structs (x86-64)
    assert C.sizeof(sam3.EncoderConfig) == 13 * 4
    assert C.sizeof(sam3.PaletteLinear) == 3 * 8 + 2 * 4
    assert C.sizeof(sam3.BlockWeights) == 2 * 8 + 2 * 32 + 2 * 8 + 2 * 32
    assert C.sizeof(sam3.EncoderWeights) == 3 * 8 + 8
    assert C.sizeof(sam3.NeckWeights) == 4 * 8 + 2 * 4
    assert C.sizeof(sam3.WindowedEncoderWeights) == 4 * 8 + 2 * 4 + 8 + 8


def test_default_config_matches_benchmark_spec(sam3):
    c = sam3.default_config()
    assert (c.embed_dim, c.num_heads, c.mlp_hidden, c.num_blocks) == (1024, 16, 4096, 32)
    assert (c.patch, c.image_size, c.prune_after_block, c.keep_tokens) == (14, 1008, 16, 2592)
    assert c.score_norm == sam3.SCORE_L2 and c.keep_order == sam3.ORDER_INDEX
    assert abs(c.ln_eps - 1e-6) < 1e-12 and c.rope_theta == 10000.0


@pytest.mark.parametrize("field,value,status", [
    ("num_heads", 8, 2),          # head_dim 128 unsupported -> SAM3_ERR_SHAPE
    ("image_size", 1000, 2),      # not a multiple of the patch
    ("score_norm", 7, 1),         # bad enum -> SAM3_ERR_INVALID_ARG
    ("keep_order", 3, 1),
    ("max_batch", 0, 2),
])
def test_ctx_create_rejects_bad_config_before_touching_a_gpu(sam3, field, value, status):
    cfg = sam3.default_config(**{field: value})
    h = C.c_void_p()
    assert sam3.lib.sam3_ctx_create(0, C.byref(cfg), C.byref(h)) == status
    assert h.value is None


def test_null_context_is_an_error_not_a_crash(sam3):
    assert sam3.lib.sam3_sync(None) == sam3.ERR_INVALID_ARG
    assert sam3.lib.sam3_ctx_destroy(None) == sam3.ERR_INVALID_ARG
    assert sam3.lib.sam3_last_error(None) == b"null context"
    assert sam3.lib.sam3_ctx_create(0, None, None) == sam3.ERR_INVALID_ARG


def test_cpp_operator_mirror_compiles_and_throws(tmp_path):
    # the header-only C++ mirror of the reference's operator classes, built
    # against the library; errors come back as sam3::SAM3Error (no GPU used)
    import shutil
    gxx = shutil.which("g++")
    if gxx is None:
        pytest.skip("no g++")
    pkg = PKG
    exe = str(tmp_path / "mirror_check")
    cmd = [gxx, "-std=c++17", "-O1", "-Wall", "-Werror",
           "-I/usr/local/cuda/include", "-I" + os.path.join(pkg, "host"),
           os.path.join(ROOT, "tests", "host_mirror_check.cpp"),
           "-L" + pkg, "-lsam3cuda", "-L/usr/local/cuda/lib64", "-lcudart",
           "-Wl,-rpath," + pkg, "-Wl,-rpath,/usr/local/cuda/lib64", "-o", exe]
    r = subprocess.run(cmd, capture_output=True, text=True)
    assert r.returncode == 0, r.stderr
    r = subprocess.run([exe], capture_output=True, text=True, timeout=60)
    assert r.returncode == 0, r.stdout + r.stderr
    assert "caught 8 of 8" in r.stdout
