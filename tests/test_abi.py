"""CPU: the C-ABI library loads, exports every symbol the header declares, and its
host-only logic (status names, argument checks, device discovery, TP share math) behaves
without a GPU."""
import ctypes
import json
import os
import re

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "magnetar_cuda.h")


def declared_functions():
    text = open(HEADER).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(mg_[a-z0-9_]+)\s*\(", text)))


def test_library_exports_every_declared_symbol(mpc):
    lib = mpc.lib()
    names = declared_functions()
    assert len(names) > 60
    missing = [n for n in names if not hasattr(lib, n)]
    assert not missing, missing


def test_binding_covers_the_header(mpc):
    from importlib import import_module
    native = import_module("magnetar-provider-cuda_b200._native")
    assert set(declared_functions()) == set(native.SIGNATURES), \
        set(declared_functions()) ^ set(native.SIGNATURES)


def test_abi_version_and_status_names(mpc):
    lib = mpc.lib()
    assert lib.mg_abi_version() == 1
    from importlib import import_module
    native = import_module("magnetar-provider-cuda_b200._native")
    for code, name in native.STATUS_NAMES.items():
        assert lib.mg_status_name(code).decode() == ("Ok" if code == 0 else name)


def test_null_arguments_are_refused(mpc):
    lib = mpc.lib()
    assert lib.mg_device_open(0, None) == 12
    assert lib.mg_buffer_upload(None, None, 0) == 12
    assert lib.mg_add(None, None, None, None) == 12
    assert b"null" in lib.mg_last_error()


def test_device_discovery_without_gpu_is_graceful(mpc):
    import torch
    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    n = ctypes.c_int(-1)
    assert mpc.lib().mg_device_count(ctypes.byref(n)) == 0 and n.value == 0
    h = ctypes.c_void_p()
    assert mpc.lib().mg_device_open(0, ctypes.byref(h)) == 8  # DeviceUnavailable
    p = mpc.CudaProvider.new()
    assert not p.is_available() and p.health() == "Unavailable"
    assert p.execution_api() is None and p.advertisements() == []


def test_advertisements_mirror_the_reference(mpc):
    ads = mpc.cuda_kernel_advertisements("cuda:0")
    names = [a.name for a in ads]
    # src/tests.rs:130-153 lists the reference's set; all but moe-experts (out of scope) here
    for n in ["matmul", "matmul-bias", "matmul-residual", "gated-matmul", "silu-mul", "embedding", "rmsnorm",
              "rope", "attention", "softmax", "silu", "add", "mul", "residual-add", "add-half", "mul-half",
              "batched-matmul", "row-scale", "activation", "kv-write", "gelu", "concat"]:
        assert n in names
    by = {a.name: a for a in ads}
    assert all(by[n].rank == 2 for n in ("matmul", "rope", "attention", "softmax"))
    assert by["add"].rank is None
    assert by["add-half"].operator == "add" and by["add-half"].input_dtypes == ("f16", "bf16")
    assert all(a.conformance_profile == "cuda-conformance-v1" and a.kernel_family == "Cuda" for a in ads)


def test_tp_shares_match_reference_vectors(mpc):
    from importlib import import_module
    tp = import_module("magnetar-provider-cuda_b200.tensor_parallel")
    g = json.load(open(os.path.join(ROOT, "tests", "golden", "tp_shares.json")))
    for extent, parts, expect in g["share_granule"]:
        assert tp.share_granule(extent, parts) == expect
    for extent, parts, member, expect in g["local_extent"]:
        s, e = tp.share(extent, parts, member)
        assert e - s == expect
        assert tp.native_share(extent, parts, member) == (s, e)
    t = np.arange(12, dtype=np.float32).reshape(2, 6)
    assert tp.split_columns(t, 2, 0).reshape(-1).tolist() == g["split_2x6"]["columns"][0]
    assert tp.split_columns(t, 2, 1).reshape(-1).tolist() == g["split_2x6"]["columns"][1]
    assert tp.split_rows(t, 2, 0).reshape(-1).tolist() == g["split_2x6"]["rows0"]
    assert tp.split_columns(np.arange(6, dtype=np.float32), 2, 1).tolist() == g["split_2x6"]["bias_columns1"]
    for member, rng in enumerate(g["expert_range_5_of_2"]):
        assert list(tp.share(5, 2, member)) == rng


@pytest.mark.parametrize("extent,parts", [(28672, 8), (28672, 2), (1376, 4), (100, 3), (7, 8), (0, 2)])
def test_tp_shares_tile_the_extent(mpc, extent, parts):
    from importlib import import_module
    tp = import_module("magnetar-provider-cuda_b200.tensor_parallel")
    ends = [tp.share(extent, parts, m) for m in range(parts)]
    assert ends[0][0] == 0 and ends[-1][1] == extent
    assert all(ends[i][1] == ends[i + 1][0] for i in range(parts - 1))
    assert all(tp.native_share(extent, parts, m) == ends[m] for m in range(parts))


def test_torch_imports_after_the_library_in_a_fresh_process():
    # The library links libnccl.so.2 by its soname; loading it first must not leave an older
    # system NCCL in place of the one torch was built against (torch's import then fails).
    import subprocess
    import sys
    code = ("import importlib, sys; sys.path.insert(0, sys.argv[1]); "
            "importlib.import_module('magnetar-provider-cuda_b200._native').lib(); import torch; print('ok')")
    res = subprocess.run([sys.executable, "-c", code, ROOT], capture_output=True, text=True, timeout=300)
    assert res.returncode == 0 and res.stdout.strip().endswith("ok"), res.stderr[-2000:]
