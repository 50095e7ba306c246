"""The allocation-free MLA decode entry point, called through its exported C
symbol the way a host runtime that owns all device memory would call it
(such a caller cannot let a library cudaMalloc scratch space).  Its output
must match the regular entry point (which takes caller-allocated scratch)
on two calls in a row, since the second call reuses the library's fixed
scratch arrays with the first call's contents still in them.

This file sorts last so that a run stopping at the first failure has
already run every other test."""
import ctypes
import os

import pytest
import torch

pytestmark = pytest.mark.gpu

DEV = "cuda"
ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _lib():
    import b200ds._C as ext  # the regular entry points live in the same library
    lib = ctypes.CDLL(ext.__file__)
    fn = lib.b200_mla_decode_noalloc
    fn.restype = ctypes.c_int
    fn.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int, ctypes.c_int, ctypes.c_void_p, ctypes.c_longlong,
                   ctypes.c_void_p, ctypes.c_int, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int, ctypes.c_float,
                   ctypes.c_float, ctypes.c_int, ctypes.c_void_p, ctypes.c_void_p]
    err = lib.b200_mla_decode_noalloc_error
    err.restype = ctypes.c_char_p
    err.argtypes = [ctypes.c_int]
    return fn, err


def _status():
    import b200ds._C as ext
    st = ctypes.CDLL(ext.__file__).b200_mla_decode_noalloc_status
    st.restype = ctypes.c_int
    st.argtypes = [ctypes.c_void_p, ctypes.POINTER(ctypes.c_uint)]
    word = ctypes.c_uint(0xFFFFFFFF)
    rc = st(torch.cuda.current_stream().cuda_stream, ctypes.byref(word))
    return rc, word.value


def _case(seed, T=8, H=16, ps=64):
    g = torch.Generator().manual_seed(seed)
    lens = torch.randint(70, 900, (T,), generator=g).tolist()
    pages = [(n + ps - 1) // ps for n in lens]
    mp = max(pages)
    bt = torch.zeros(T, mp, dtype=torch.int32)
    nxt = 1
    for b in range(T):
        for j in range(pages[b]):
            bt[b, j] = nxt
            nxt += 1
    cache = (torch.randn(nxt * ps, 576, generator=g) * 0.5).to(torch.float8_e4m3fn)
    q_abs = (torch.randn(T, H, 512, generator=g) * 0.3).to(torch.bfloat16)
    q_pe = (torch.randn(T, H, 64, generator=g) * 0.3).to(torch.bfloat16)
    q_seq = torch.arange(T, dtype=torch.int32)
    q_pos = torch.tensor([n - 1 for n in lens], dtype=torch.int32)
    return [t.to(DEV) for t in (q_abs, q_pe, cache, bt, q_seq, q_pos)]


def _regular(q_abs, q_pe, cache, bt, q_seq, q_pos, nsplit, sm, kvs):
    from b200ds import _C
    T, H, L = q_abs.shape
    q8 = torch.empty(T, H, 576, dtype=torch.uint8, device=DEV)
    qs = torch.empty(T, H, dtype=torch.float32, device=DEV)
    _C.mla_q_quant(q_abs, q_pe, q8, qs)
    out = torch.empty(T, H, L, dtype=torch.bfloat16, device=DEV)
    po = torch.empty(nsplit, T, H, L, dtype=torch.float32, device=DEV)
    pl = torch.empty(nsplit, T, H, dtype=torch.float32, device=DEV)
    _C.mla_tc(q8, qs, cache.view(torch.uint8), kvs, bt, q_seq, q_pos, 64, sm, nsplit, out, po, pl)
    return out


def test_noalloc_entry_point_matches_regular_entry_point_twice():
    fn, err = _lib()
    stream = torch.cuda.current_stream().cuda_stream
    sm, kvs, nsplit = 0.0625, 0.7, 3
    for seed in (0, 1):   # two calls in a row: the second reuses the scratch
        q_abs, q_pe, cache, bt, q_seq, q_pos = _case(seed)
        T, H, _ = q_abs.shape
        out = torch.full((T, H, 512), float("nan"), dtype=torch.bfloat16, device=DEV)
        rc = fn(q_abs.data_ptr(), q_pe.data_ptr(), T, H, cache.data_ptr(), cache.shape[0], bt.data_ptr(), bt.stride(0),
                q_seq.data_ptr(), q_pos.data_ptr(), 64, sm, kvs, nsplit, out.data_ptr(), stream)
        assert rc == 0, err(rc).decode()
        exp = _regular(q_abs, q_pe, cache, bt, q_seq, q_pos, nsplit, sm, kvs)
        torch.cuda.synchronize()
        # same kernels, same inputs, same split count: bit-identical output,
        # and no NaN of the NaN-filled output buffer survives
        assert not torch.isnan(out.float()).any()
        assert torch.equal(out, exp)
        rc, word = _status()     # every wait of the call finished in time
        assert rc == 0 and word == 0, (rc, word)


def test_noalloc_entry_point_rejects_oversized_requests():
    fn, err = _lib()
    q_abs, q_pe, cache, bt, q_seq, q_pos = _case(2)
    T, H, _ = q_abs.shape
    out = torch.empty(T, H, 512, dtype=torch.bfloat16, device=DEV)
    # 8 tokens x 16 heads x 16 splits = 2048 partial rows fits; 600 tokens x 16 heads does not
    rc = fn(q_abs.data_ptr(), q_pe.data_ptr(), 600, 16, cache.data_ptr(), cache.shape[0], bt.data_ptr(), bt.stride(0),
            q_seq.data_ptr(), q_pos.data_ptr(), 64, 0.1, 1.0, 1, out.data_ptr(), torch.cuda.current_stream().cuda_stream)
    assert rc == -2 and b"static scratch" in err(rc)
