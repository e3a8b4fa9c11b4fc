"""Shared test setup: the ``gpu`` marker, repo import path and golden-fixture loaders."""
import sys
from pathlib import Path

import numpy as np
import pytest
import torch

REPO = Path(__file__).resolve().parent.parent
GOLDEN = Path(__file__).resolve().parent / "golden"
if str(REPO) not in sys.path:
    sys.path.insert(0, str(REPO))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100) GPU and the built libhyb200.so")


def load_golden(name: str) -> dict:
    with np.load(GOLDEN / name, allow_pickle=False) as z:
        return {k: z[k] for k in z.files}


def bf16(a: np.ndarray) -> torch.Tensor:
    """int16 bit patterns -> bf16 tensor."""
    return torch.from_numpy(np.ascontiguousarray(a)).view(torch.bfloat16)


def e4m3(a: np.ndarray) -> torch.Tensor:
    return torch.from_numpy(np.ascontiguousarray(a)).view(torch.float8_e4m3fn)


@pytest.fixture(scope="session")
def cuda_lib():
    """The built library on an sm_100 device (GPU tests only)."""
    from hy_nomas_b200 import _lib
    if not torch.cuda.is_available():
        pytest.fail("GPU test run without a CUDA device")
    lib = _lib.load()
    assert lib.hyb_device_supported() == 1, "libhyb200 needs an sm_100 device"
    return lib


def config1_inputs():
    """The seeded BASELINE config-1 inputs (hist_k, hist_v, [img_q, img_k, img_v, txt_q,
    txt_k, txt_v]) exactly as tests/golden/make_golden.py generated them for attn_config1.npz."""
    import importlib.util
    spec = importlib.util.spec_from_file_location("make_golden", GOLDEN / "make_golden.py")
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    hk, hv, cur = mod.config1_inputs()
    return hk, hv, cur, mod.input_checksums([hk, hv, *cur])


def intra_case(name):
    """Inputs of an intra-segment fixture: decoded history, the chunk, masks, per-sample
    offsets (None where the reference got None) and the windows in tokens."""
    g = load_golden(f"intra_{name}.npz")
    Lh, T = int(g["Lh"]), int(g["T"])
    counts, flat = g["offsets"].tolist(), g["offsets_flat"].tolist()
    offsets, pos = [], 0
    for c in counts:
        offsets.append(None if c < 0 else flat[pos:pos + c])
        pos += max(c, 0)
    windows = [[int(a) * T, int(b) * T, int(c)] for a, b, c in g["windows"].tolist()]
    from oracle import quant as oq
    hk = oq.dequantize(torch.from_numpy(g["hist_k"][:, :Lh]), torch.from_numpy(g["hist_k_scale"][:, :Lh]))
    hv = oq.dequantize(torch.from_numpy(g["hist_v"][:, :Lh]), torch.from_numpy(g["hist_v_scale"][:, :Lh]))
    cur = [bf16(g[n]) for n in ("img_q", "img_k", "img_v", "txt_q", "txt_k", "txt_v")]
    return g, Lh, T, offsets, windows, hk, hv, cur
