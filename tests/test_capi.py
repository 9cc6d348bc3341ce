"""CPU checks of the C ABI: the library loads, exports every symbol that
include/moe_b200.h declares, and rejects bad arguments before touching a GPU.
No kernel is launched here."""
import ctypes
import re
from ctypes import byref, c_size_t

import pytest

from conftest import PKG, ROOT


@pytest.fixture(scope="module")
def lib():
    import moe_b200
    from moe_b200 import build
    build.build()
    return moe_b200.load_library()


def header_symbols():
    text = (ROOT / "include" / "moe_b200.h").read_text()
    return set(re.findall(r"^\s*(?:int|const char\*)\s+(moe_\w+)\s*\(", text, re.M))


def test_header_symbols_exported(lib):
    syms = header_symbols()
    assert len(syms) >= 15
    for s in syms:
        assert hasattr(lib, s), s
    from moe_b200 import _lib
    assert syms == set(_lib.EXPORTED)


def test_abi_version(lib):
    assert lib.moe_b200_abi_version() == 2


def test_workspace_sizes(lib):
    n = c_size_t(0)
    assert lib.moe_row_id_map_workspace_size(16384, 256, byref(n)) == 0
    assert n.value >= 256 * 256 * 4 and n.value % 256 == 0
    assert lib.moe_grouped_gemm_workspace_size(256, byref(n)) == 0
    assert n.value >= 256 + 4 * 256 * 4
    assert lib.moe_grouped_gemm_workspace_size(0, byref(n)) == 1
    assert b"out of range" in lib.moe_b200_last_error()


def test_invalid_arguments_are_rejected_without_launch(lib):
    # odd row pointer (rows move in 2-byte units at least)
    assert lib.moe_permute_mask_map(17, 16, None, 32, None, 4, 12, 2, 4, None) == 1
    assert b"aligned" in lib.moe_b200_last_error()
    # null rows
    assert lib.moe_permute_mask_map(None, None, None, None, None, 4, 12, 2, 4, None) == 1
    assert b"null" in lib.moe_b200_last_error()
    # probs without permuted_probs
    assert lib.moe_permute_mask_map(16, 16, 16, 16, None, 4, 8, 2, 4, None) == 1
    assert b"both" in lib.moe_b200_last_error()
    # bad idx_bits
    assert lib.moe_unpermute_mask(None, None, 16, None, 0, None, None, 4, 8, 2, 4, None) == 1
    # k beyond this build
    assert lib.moe_topk_f32(16, 16, 16, 4, 64, 17, None) == 2
    # empty shapes are no-ops that succeed without a device
    assert lib.moe_permute_mask_map(None, None, None, None, None, 0, 8, 2, 0, None) == 0
    assert lib.moe_topk_f32(16, 16, 16, 0, 64, 8, None) == 0
    # GEMM argument checks
    assert lib.moe_grouped_gemm(None, None, None, 10, 4, 4, 256, 12, 0, None, 0, None) == 1
    assert lib.moe_grouped_gemm(None, None, None, 10, 4, 4, 256, 64, 2, None, 0, None) == 1
    # fused router: E must be a multiple of 32 up to 512, 1 <= k <= 16, an
    # error word is required, and at least one output must be asked for
    rg = lib.moe_router_gemm_topk
    assert rg(16, 16, None, 16, 64, 48, 4, 1, 1, None, None, None, 16, 16, 16, None) == 1
    assert b"multiple of 32" in lib.moe_b200_last_error()
    assert rg(16, 16, None, 16, 64, 1024, 4, 1, 1, None, None, None, 16, 16, 16, None) == 1
    assert rg(16, 16, None, 16, 64, 64, 17, 1, 1, None, None, None, 16, 16, 16, None) == 1
    assert rg(16, 16, None, 16, 64, 64, 4, 1, 1, None, None, None, 16, 16, None, None) == 1
    assert b"device_error" in lib.moe_b200_last_error()
    assert rg(16, 16, None, 16, 64, 64, 4, 1, 1, None, None, None, None, None, 16, None) == 1
    assert b"no output" in lib.moe_b200_last_error()
    assert rg(16, 16, None, 16, 60, 64, 4, 1, 1, None, None, None, 16, 16, 16, None) == 1
    assert rg(16, 16, None, 16, 64, 64, 4, 2, 1, None, None, None, 16, 16, 16, None) == 1
    assert rg(None, None, None, 0, 64, 64, 4, 1, 1, None, None, None, None, None, 16, None) == 0
    # backward of the combine and of SwiGLU
    cb = lib.moe_combine_backward
    assert cb(16, 16, 16, 16, 16, 16, 4, 8, 2048, 8, None) == 1  # E above 1024
    assert cb(None, None, None, None, None, None, 4, 8, 4, 8, None) == 1  # null pointers
    assert cb(None, None, None, None, None, None, 0, 8, 4, 0, None) == 0  # no tokens
    sb = lib.moe_swiglu_backward
    assert sb(16, 16, 16, 4, 12, None) == 1  # F not a multiple of 8
    assert b"multiple of 8" in lib.moe_b200_last_error()
    assert sb(17, 16, 16, 4, 16, None) == 1  # misaligned
    assert sb(None, None, None, 0, 16, None) == 0
    # grouped wgrad: host counts travel in the launch (G <= 4096); device
    # counts need a pointer
    wg = lib.moe_grouped_wgrad
    assert wg(16, 16, 16, 10, 5000, 64, 64, 16, 256, 1 << 30, None) == 1
    assert b"4096" in lib.moe_b200_last_error()
    assert lib.moe_grouped_wgrad_dev(16, 16, 16, 10, 8, 64, 64, None, 256, 1 << 30, None) == 1
    assert b"device array" in lib.moe_b200_last_error()
    # permute from the expert list: 1 <= k <= 32, 16-byte rows
    pt = lib.moe_permute_topk
    assert pt(16, 16, 16, 33, None, 16, None, 4, 64, 8, 32, None) == 1
    assert pt(16, 16, 16, 4, None, 16, None, 4, 60, 8, 32, None) == 1
    assert pt(None, None, None, 4, None, None, None, 0, 64, 8, 0, None) == 0
    # pull dispatch: groups a multiple of the ranks and at most 1024, 16-byte rows
    pb = (ctypes.c_int64 * 2)(256, 512)
    pd = lib.moe_ep_dispatch_pull
    assert pd(pb, pb, 2, 64, 512, 16, 3, 256, 10, 100, 64, None) == 1
    assert b"multiple of ranks" in lib.moe_b200_last_error()
    assert pd(pb, pb, 2, 64, 512, 16, 2048, 256, 10, 100, 64, None) == 1
    assert pd(pb, pb, 2, 64, 512, 16, 4, 256, 10, 100, 60, None) == 1
    assert pd(pb, pb, 2, 64, 512, 16, 4, 256, 0, 100, 64, None) == 0  # nothing to receive
    assert lib.moe_ep_pull_stage(16, 16, 4, 60, 8, 32, 16, 16, None) == 1
    assert lib.moe_ep_pull_stage(None, None, 0, 64, 8, 0, None, None, None) == 0
    # one chunk of the fused EP dispatch: the local expert range must lie in
    # [0, experts_per_rank); an empty range launches nothing
    dr = lib.moe_ep_dispatch_range
    bases = (ctypes.c_int64 * 2)(256, 512)
    assert dr(16, 16, bases, 16, 2, 4, 64, 8, 64, 8, 32, 3, 5, 0, None) == 1
    assert b"local expert range" in lib.moe_b200_last_error()
    assert dr(16, 16, bases, 16, 2, 4, 64, 8, 64, 8, 32, 2, 1, 0, None) == 1
    assert dr(16, 16, bases, 16, 2, 4, 64, 8, 64, 8, 32, 0, 2, -1, None) == 1
    assert dr(16, 16, bases, 16, 2, 4, 64, 8, 64, 8, 32, 2, 2, 0, None) == 0


def test_ops_refuse_cpu_tensors():
    import torch
    import moe_b200
    with pytest.raises(ValueError):
        moe_b200.topk(torch.randn(4, 8), 2)
    with pytest.raises(ValueError):
        moe_b200.permute(torch.zeros(4, 8, dtype=torch.bfloat16),
                         torch.zeros(4, 2, dtype=torch.int64))
    with pytest.raises(ValueError):
        moe_b200.grouped_gemm(torch.zeros(4, 8, dtype=torch.bfloat16),
                              torch.zeros(1, 8, 8, dtype=torch.bfloat16))
    x16 = torch.zeros(4, 64, dtype=torch.bfloat16)
    w16 = torch.zeros(32, 64, dtype=torch.bfloat16)
    with pytest.raises(ValueError):
        moe_b200.router_gemm_topk(x16, w16, 4)
    with pytest.raises(ValueError):
        moe_b200.router_logits(x16, w16)
    with pytest.raises(ValueError):
        moe_b200.grouped_wgrad(torch.zeros(4, 8, dtype=torch.bfloat16),
                               torch.zeros(4, 8, dtype=torch.bfloat16), [4])
    with pytest.raises(ValueError):
        moe_b200.permute_backward(torch.zeros(4, 8, dtype=torch.bfloat16),
                                  torch.zeros(2, 4, dtype=torch.int64))
    with pytest.raises(ValueError):
        moe_b200.combine_backward(torch.zeros(4, 8, dtype=torch.bfloat16),
                                  torch.zeros(8, 8, dtype=torch.bfloat16),
                                  torch.zeros(4, 2, dtype=torch.int64), torch.zeros(4, 2))
    with pytest.raises(ValueError):
        moe_b200.swiglu_backward(torch.zeros(4, 16, dtype=torch.bfloat16),
                                 torch.zeros(4, 8, dtype=torch.bfloat16))


def test_product_package_does_not_import_oracle():
    pat = re.compile(r"^\s*(from\s+oracle\b|import\s+oracle\b)|moe_oracle", re.M)
    for p in PKG.rglob("*.py"):
        assert not pat.search(p.read_text()), p


def test_plain_c_consumer(lib, tmp_path):
    """The header and library are usable from C alone: gcc compiles
    tests/capi_consumer.c against include/moe_b200.h (no CUDA headers) and
    links the built library; the program checks calls that need no GPU."""
    import shutil
    import subprocess
    gcc = shutil.which("gcc")
    if gcc is None:
        pytest.skip("gcc not available")
    libdir = PKG / "lib"
    exe = tmp_path / "capi_consumer"
    subprocess.run([gcc, "-std=c99", "-Wall", "-Werror", f"-I{ROOT / 'include'}",
                    str(ROOT / "tests" / "capi_consumer.c"), f"-L{libdir}", "-lmoe_b200",
                    f"-Wl,-rpath,{libdir}", "-o", str(exe)], check=True, timeout=120)
    r = subprocess.run([str(exe)], capture_output=True, text=True, timeout=60)
    assert r.returncode == 0 and "C consumer OK" in r.stdout, r.stdout + r.stderr
