"""The allocation-free C entry point of the attention decode (``csrc/noalloc.h``).

Calls ``isb_attention_decode_noalloc`` through its exported C symbol (ctypes on
the in-tree extension) and compares it with the PyTorch-facing
``torch.ops.isb.attention_decode`` on two calls in a row with different
shapes, so the second call runs over scratch the first one left behind.
"""

import ctypes

import pytest
import torch

pytestmark = pytest.mark.gpu

OK, ETOOBIG, EINVAL = 0, 1, 3
SCRATCH_BYTES = 16 << 20


def _lib():
    from inference_systems_b200.ops._ext import load_extension

    load_extension()
    import inference_systems_b200._C as ext

    lib = ctypes.CDLL(ext.__file__)
    f = lib.isb_attention_decode_noalloc
    f.restype = ctypes.c_int
    f.argtypes = [ctypes.c_void_p] * 4 + [ctypes.c_void_p, ctypes.c_void_p] + [ctypes.c_int] * 5 + \
        [ctypes.c_float, ctypes.c_void_p, ctypes.c_void_p]
    lib.isb_attention_decode_noalloc_scratch_bytes.restype = ctypes.c_size_t
    lib.isb_attention_decode_noalloc_scratch_bytes.argtypes = [ctypes.c_int] * 4
    lib.isb_noalloc_strerror.restype = ctypes.c_char_p
    lib.isb_noalloc_strerror.argtypes = [ctypes.c_int]
    lib.isb_noalloc_setup.restype = ctypes.c_int
    lib.isb_noalloc_error_word.restype = ctypes.c_uint
    lib.isb_noalloc_error_word.argtypes = []
    return lib


def _case(b, hq, hkv, hd, ctx, max_blocks, seed):
    g = torch.Generator(device="cuda").manual_seed(seed)
    dev, bf = "cuda", torch.bfloat16
    nblocks = b * max_blocks + 3
    kc = torch.randn(nblocks, hkv, 256, hd, device=dev, generator=g).to(bf)
    vc = torch.randn(nblocks, hkv, 256, hd, device=dev, generator=g).to(bf)
    q = torch.randn(b, hq, hd, device=dev, generator=g).to(bf)
    gate = torch.randn(b, hq * hd, device=dev, generator=g).to(bf)
    perm = torch.randperm(nblocks, device=dev, generator=g)[: b * max_blocks].to(torch.int32)
    bt = perm.view(b, max_blocks).contiguous()
    cl = torch.tensor(ctx, dtype=torch.int32, device=dev)
    return q, gate, kc, vc, cl, bt


def _call(lib, q, gate, kc, vc, cl, bt, scale, out):
    b, hq, hd = q.shape
    code = lib.isb_attention_decode_noalloc(
        q.data_ptr(), gate.data_ptr() if gate is not None else None, kc.data_ptr(), vc.data_ptr(),
        cl.data_ptr(), bt.data_ptr(), bt.shape[1], b, hq, kc.shape[1], hd, scale, out.data_ptr(),
        torch.cuda.current_stream().cuda_stream)
    return code


def test_noalloc_decode_matches_allocating_entry_point():
    lib = _lib()
    assert lib.isb_noalloc_setup() == OK
    cases = [
        # (batch, q heads, kv heads, head_dim, context lengths, max_blocks, gated)
        (8, 8, 2, 256, [1, 63, 64, 65, 300, 512, 640, 200], 3, True),
        (5, 4, 2, 128, [700, 9, 256, 257, 1000], 4, False),
    ]
    for i, (b, hq, hkv, hd, ctx, mb, gated) in enumerate(cases):
        q, gate, kc, vc, cl, bt = _case(b, hq, hkv, hd, ctx, mb, seed=10 + i)
        scale = hd ** -0.5
        gate_arg = gate if gated else torch.empty(0, hq * hd, device="cuda", dtype=torch.bfloat16)
        want = torch.ops.isb.attention_decode(q, gate_arg, kc, vc, cl, bt, scale, gated)
        out = torch.full((b, hq * hd), float("nan"), device="cuda", dtype=torch.bfloat16)
        torch.cuda.synchronize()
        before = torch.cuda.memory_allocated()
        free_before = torch.cuda.mem_get_info()[0]
        code = _call(lib, q, gate if gated else None, kc, vc, cl, bt, scale, out)
        torch.cuda.synchronize()
        assert code == OK, lib.isb_noalloc_strerror(code).decode()
        assert torch.cuda.memory_allocated() == before
        # a cudaMalloc inside the call would take device memory outside PyTorch's allocator
        assert torch.cuda.mem_get_info()[0] == free_before
        assert torch.isfinite(out.float()).all()
        torch.testing.assert_close(out.float(), want.float(), atol=2e-2, rtol=2e-2)
    assert lib.isb_noalloc_error_word() == 0
    assert torch.ops.isb.error_word() == 0


def test_noalloc_context_past_block_table_is_flagged():
    """A context one page longer than the block table: finite output over the pages it has, and
    the error word (read through the C API) says the call's output is not valid."""
    lib = _lib()
    assert lib.isb_noalloc_setup() == OK
    assert lib.isb_noalloc_error_word() == 0
    b, hq, hkv, hd, mb = 2, 8, 2, 256, 2
    q, gate, kc, vc, cl, bt = _case(b, hq, hkv, hd, [100, mb * 256 + 256], mb, seed=31)
    out = torch.full((b, hq * hd), float("nan"), device="cuda", dtype=torch.bfloat16)
    code = _call(lib, q, gate, kc, vc, cl, bt, hd ** -0.5, out)
    torch.cuda.synchronize()
    assert code == OK, lib.isb_noalloc_strerror(code).decode()
    assert torch.isfinite(out.float()).all()
    assert lib.isb_noalloc_error_word() == 0x2
    assert lib.isb_noalloc_error_word() == 0  # read-and-clear
    # the in-range sequence is unaffected
    want = torch.ops.isb.attention_decode(q[:1], gate[:1], kc, vc, cl[:1], bt[:1], hd ** -0.5, True)
    torch.testing.assert_close(out[:1].float(), want.float(), atol=2e-2, rtol=2e-2)


def test_noalloc_rejects_oversized_and_invalid():
    lib = _lib()
    need = lib.isb_attention_decode_noalloc_scratch_bytes(4096, 64, 256, 64)
    assert need > SCRATCH_BYTES
    # Null pointers with oversized shapes: the size check answers before any pointer is used.
    code = lib.isb_attention_decode_noalloc(None, None, None, None, None, None, 64, 4096, 64, 8, 256, 1.0, None, None)
    assert code == ETOOBIG
    assert b"scratch" in lib.isb_noalloc_strerror(code)
    code = lib.isb_attention_decode_noalloc(None, None, None, None, None, None, 3, 8, 8, 2, 256, 1.0, None, None)
    assert code == EINVAL
    # a block table wider than the decode grid can cover is invalid, not an int overflow
    code = lib.isb_attention_decode_noalloc(None, None, None, None, None, None, 1 << 29, 1, 8, 2, 256, 1.0, None, None)
    assert code == EINVAL
    # The largest batch of the 0.8B decode shape (8 q heads, head_dim 256, 3 pages) fits.
    assert lib.isb_attention_decode_noalloc_scratch_bytes(128, 8, 256, 3) <= SCRATCH_BYTES
