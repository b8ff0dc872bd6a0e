"""tq4_matmul_noalloc: the allocation-free decode call, for callers that cannot call cudaMalloc
(a NIF next to EXLA's preallocating CUDA client, or a decode loop that must not risk the device
synchronization of cudaMalloc/cudaFree). Its split-K scratch is a static device array shared by
all calls, so these tests check two calls in a row against tq4_matmul, with the tolerance the
other parity tests use, plus the size limit. The file is named so pytest collects it last."""

import ctypes

import numpy as np
import pytest
import torch

from oracle import matmul_nbits as o
from transmuter_b200 import _lib, workloads
from transmuter_b200.quantized import TORCH_TO_TQ4, PackedWeight

pytestmark = pytest.mark.gpu

DEV = "cuda:0"
TOL = {torch.float32: 1e-3, torch.float16: 5e-3, torch.bfloat16: 5e-3}


def noalloc(w, a, bias=None, out_dtype=None):
    lib = _lib.load()
    lib.tq4_matmul_noalloc.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int64, ctypes.c_int,
                                       ctypes.c_void_p, ctypes.c_int, ctypes.c_void_p, ctypes.c_int,
                                       ctypes.c_void_p]
    lib.tq4_matmul_noalloc.restype = ctypes.c_int
    y = torch.empty((a.shape[0], w.n), dtype=out_dtype or a.dtype, device=a.device)
    st = lib.tq4_matmul_noalloc(w._handle, ctypes.c_void_p(a.data_ptr()), a.shape[0], TORCH_TO_TQ4[a.dtype],
                                ctypes.c_void_p(bias.data_ptr()) if bias is not None else None,
                                TORCH_TO_TQ4[bias.dtype] if bias is not None else 0,
                                ctypes.c_void_p(y.data_ptr()), TORCH_TO_TQ4[y.dtype],
                                ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    return st, y


def make_weight(cfg):
    p = workloads.make(cfg)
    tt = {"f32": torch.float32, "f16": torch.float16, "bf16": torch.bfloat16}
    w = PackedWeight((cfg.k, cfg.n, cfg.bits, cfg.block_size), torch.from_numpy(p["B"]).to(DEV),
                     torch.from_numpy(p["scales"]).to(DEV),
                     torch.from_numpy(p["zp"]).to(DEV) if p["zp"] is not None else None,
                     dtype=tt[cfg.scale_type], device=DEV)
    return w, p


@pytest.mark.parametrize("name,m", [("c5-4096x1024-m16", 16), ("c5-4096x1024-m1", 1), ("c5-14336x4096-m16", 16),
                                    ("c1", 1), ("c5-4096x14336-m16", 9), ("c3m1", 1)])
def test_noalloc_matches_matmul_on_two_calls(name, m):
    cfg = workloads.CONFIGS[name]
    w, p = make_weight(cfg)
    tt = torch.float16 if cfg.a_type == "f16" else torch.float32
    a = torch.from_numpy(np.asarray(p["A"][:m])).to(DEV, tt)
    a2 = torch.flip(a, dims=[1]).contiguous()  # a different second input: no stale result passes
    for x in (a, a2):
        st, y = noalloc(w, x)
        assert st == 0, _lib.last_error()
        ref = w.matmul(x)
        torch.cuda.synchronize()
        err = o.rel_l2(y.float().cpu().numpy(), ref.float().cpu().numpy())
        assert err < TOL[tt], err
        assert torch.isfinite(y).all()


def test_noalloc_rejects_beyond_its_limits():
    cfg = workloads.Config("noalloc-too-big", 8192, 16384, 16, block_size=128, scale_type="f16", zp="packed",
                           a_type="f16")
    w, p = make_weight(cfg)
    a = torch.zeros((16, cfg.k), dtype=torch.float16, device=DEV)
    st, _ = noalloc(w, a)
    assert st == 1 and "static limit" in _lib.last_error()
    st, _ = noalloc(w, torch.zeros((17, cfg.k), dtype=torch.float16, device=DEV))
    assert st == 2 and "M <= 16" in _lib.last_error()
    y = w.matmul(a)  # the allocating entry point still takes it
    torch.cuda.synchronize()
    assert torch.count_nonzero(y) == 0


def device_status():
    code = ctypes.c_int32()
    _lib.check(_lib.load().tq4_device_status(0, ctypes.byref(code)))
    return code.value


@pytest.mark.parametrize("k,n,m,bias,at,out", [
    (4096, 4096, 4, True, torch.float16, torch.float16),    # 2 <= M <= 8 with a bias
    (4096, 1024, 3, False, torch.float16, torch.float32),   # f32 output from f16 activations
    (1024, 3072, 6, True, torch.float32, torch.float16),    # f16 output from f32 activations
    (14336, 4096, 2, True, torch.float16, torch.float16),   # split-K over the long K
])
def test_noalloc_bias_out_dtype_and_status(k, n, m, bias, at, out):
    st_name = "f16" if at == torch.float16 else "f32"
    cfg = workloads.Config(f"noalloc-{k}-{n}-{m}-{bias}-{at}-{out}", k, n, m, block_size=128 if k >= 4096 else 32,
                           scale_type=st_name, zp="packed" if k >= 4096 else "none", a_type=st_name, bias=bias)
    w, p = make_weight(cfg)
    a = torch.from_numpy(np.asarray(p["A"][:m])).to(DEV, at)
    b = torch.from_numpy(np.asarray(p["bias"])).to(DEV, at) if bias else None
    assert device_status() == 0
    for x in (a, -a):  # two calls in a row through the shared scratch
        st, y = noalloc(w, x, b, out_dtype=out)
        assert st == 0, _lib.last_error()
        ref = w.matmul(x, b, out_dtype=out)
        torch.cuda.synchronize()
        assert y.dtype == out
        err = o.rel_l2(y.double().cpu().numpy(), ref.double().cpu().numpy())
        assert err < TOL[at], err
        assert device_status() == 0
