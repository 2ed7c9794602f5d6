"""The C ABI boundary, checked without a GPU: every function declared in
include/ttk.h and include/tt_trainer.h is exported by the built libraries and
bound in the ctypes layer; the libraries load on a host without a device and
refuse to compute there (no CPU path); the C++ API headers compile, and the
reference's own model.cpp / apps/train.cpp compile against them unchanged."""
import os
import re
import shutil
import subprocess

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared(header):
    src = open(os.path.join(ROOT, "include", header)).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return sorted(set(re.findall(r"^\s*(?:const\s+)?\w+\**\s+\**((?:ttk|tt)_\w+)\s*\(", src,
                                 flags=re.M)))


def test_ttk_exports_every_declared_symbol():
    from tinytrain_b200 import _ttk
    names = declared("ttk.h")
    assert len(names) > 50
    lib = _ttk.lib()
    missing = [n for n in names if getattr(lib, n, None) is None]
    assert not missing, missing
    unbound = [n for n in names if n not in _ttk.SIGS]
    assert not unbound, unbound


def test_trainer_exports_every_declared_symbol():
    from tinytrain_b200 import trainer
    names = declared("tt_trainer.h")
    lib = trainer.lib()
    missing = [n for n in names if getattr(lib, n, None) is None]
    assert not missing, missing


def test_no_cpu_path():
    import torch
    if torch.cuda.is_available():
        pytest.skip("device present")
    from tinytrain_b200 import _ttk
    with pytest.raises(_ttk.TtkError):
        _ttk.call("ttk_init", 0)
    from tinytrain_b200.trainer import Trainer, TrainerError
    with pytest.raises(TrainerError, match="device|CUDA|cuda"):
        Trainer(dict(vocab=16, dim=8, layers=1, heads=2, ffn=16, max_seq=8), host_init=False)


def test_bucket_plan_host_logic():
    """DP gradient arena: reverse parameter order, 256-byte aligned slices,
    buckets contiguous, covering every parameter exactly once."""
    from tinytrain_b200.trainer import plan_buckets
    sizes = [32000 * 256, 256, 65536, 65536, 65536, 65536, 256, 196608, 196608, 196608, 256]
    offs, ids, buckets = plan_buckets(sizes, 1 << 20)
    order = sorted(range(len(sizes)), key=lambda i: offs[i])
    assert order == list(reversed(range(len(sizes))))
    assert all(o % 64 == 0 for o in offs)
    end = 0
    for b, (bo, bc) in enumerate(buckets):
        assert bo == end
        members = [i for i in range(len(sizes)) if ids[i] == b]
        assert members
        assert all(bo <= offs[i] < bo + bc for i in members)
        end = bo + bc
    assert end >= sum(sizes)


def test_gemm_dispatch_host_logic():
    """Host-side GEMM planning, which needs no device (148 SMs assumed when
    none is visible): exact fp32 for problems of at most 2^24 multiply-adds,
    split-K slice counts for the weight gradients of the 1B layer at 16 x 2048
    tokens (K = 32768), none for GEMMs that fill the machine, and a workspace
    that grows by the partial products when split."""
    import torch
    if torch.cuda.is_available():
        pytest.skip("the device's own SM count would apply")
    from tinytrain_b200 import _ttk
    assert _ttk.call("ttk_gemm_get_fp32_max_macs") == 1 << 24
    assert _ttk.call("ttk_gemm_uses_fp32", 1, 4, 5, 3) == 1
    assert _ttk.call("ttk_gemm_uses_fp32", 1, 32768, 2048, 2048) == 0
    assert _ttk.call("ttk_gemm_get_split_k") == 1
    assert _ttk.call("ttk_gemm_get_cta_pairs") == 1
    # dW = dY^T X: (transA, transB) = (1, 0)
    assert _ttk.call("ttk_gemm_split_k_slices", 1, 0, 1, 2048, 2048, 32768) == 8
    assert _ttk.call("ttk_gemm_split_k_slices", 1, 0, 1, 5632, 2048, 32768) == 2
    assert _ttk.call("ttk_gemm_split_k_slices", 1, 0, 1, 2048, 5632, 32768) == 2
    assert _ttk.call("ttk_gemm_split_k_slices", 1, 0, 1, 32000, 2048, 32768) == 1
    # forward / dX: plenty of tiles
    assert _ttk.call("ttk_gemm_split_k_slices", 0, 1, 1, 32768, 2048, 2048) == 1
    assert _ttk.call("ttk_gemm_split_k_slices", 0, 0, 1, 32768, 2048, 5632) == 1
    # batched problems are not split
    assert _ttk.call("ttk_gemm_split_k_slices", 1, 0, 4, 2048, 2048, 32768) == 1
    base = 2 * 2 * (2048 * 32768 + 32768 * 2048)  # bf16 hi/lo planes of A and B
    ws = _ttk.call("ttk_gemm_workspace_size", 1, 0, 1, 2048, 2048, 32768)
    assert ws >= base + 8 * 2048 * 2048 * 4
    try:
        _ttk.call("ttk_gemm_set_split_k", 0)
        assert _ttk.call("ttk_gemm_split_k_slices", 1, 0, 1, 2048, 2048, 32768) == 1
        assert _ttk.call("ttk_gemm_workspace_size", 1, 0, 1, 2048, 2048, 32768) < ws
    finally:
        _ttk.call("ttk_gemm_set_split_k", 1)
    with pytest.raises(_ttk.TtkError):
        _ttk.call("ttk_gemm_set_cta_pairs", 3)


def _gxx():
    return shutil.which("g++") and "/usr/bin/g++"


def test_cpp_api_compiles_and_links(tmp_path):
    src = tmp_path / "use_api.cpp"
    src.write_text(
        '#include "tinytrain/model.h"\n#include "tinytrain/optim.h"\n'
        "int main() { tt::GPTConfig c; c.vocab_size = 16; c.dim = 8; c.n_layers = 1;\n"
        "  c.n_heads = 2; c.ffn_dim = 16; c.max_seq_len = 8;\n"
        "  try { tt::GPTModel m(c, 1); tt::AdamW o(m.parameters(), 1e-3f);\n"
        "    auto l = tt::cross_entropy(m.forward({1,2,3,4}, 1, 4), {2,3,4,5});\n"
        "    l.backward(); o.step(); return 0; } catch (const std::exception& e) { return 3; } }\n")
    lib = os.path.join(ROOT, "tinytrain_b200", "lib")
    out = tmp_path / "use_api"
    r = subprocess.run([_gxx(), "-std=c++20", "-I" + os.path.join(ROOT, "include"), str(src),
                        "-L" + lib, "-ltinytrain", "-lttk", "-Wl,-rpath," + lib, "-o", str(out)],
                       capture_output=True, text=True)
    assert r.returncode == 0, r.stderr[-2000:]


def test_reference_model_and_train_compile_unchanged(tmp_path):
    """The reference's src/model.cpp and apps/train.cpp, unmodified, against
    this library's headers (compile only; running needs a device)."""
    from oracle import paths
    ref, nl = paths.reference_dir(), paths.nlohmann_dir()
    if not ref or not nl:
        pytest.skip("reference sources or nlohmann/json not present")
    for f in ("src/model.cpp", "apps/train.cpp"):
        r = subprocess.run([_gxx(), "-std=c++20", "-fsyntax-only", "-I" + os.path.join(ROOT, "include"),
                            "-I" + nl, os.path.join(ref, f)], capture_output=True, text=True)
        assert r.returncode == 0, (f, r.stderr[-3000:])
