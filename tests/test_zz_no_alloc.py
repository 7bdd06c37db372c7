"""The allocation-free C entry point `ad_adam_fused_noalloc`.

Some callers cannot allocate GPU memory (a host framework that owns the
memory pool, a plugin handed only raw device pointers and a stream), so the
library exports one C function that runs the fused clip + Adam update with its
scratch in a static device array. This test calls it through its exported
symbol with ctypes and checks two consecutive updates against the existing
`adam_fused` entry point, plus the rejection of a block count beyond the
scratch array's capacity. The file name sorts it last in the suite.
"""
import ctypes

import pytest
import torch

pytestmark = pytest.mark.gpu


def _lib():
    import autodrive_b200._C as ext  # loads torch's libraries and the extension
    lib = ctypes.CDLL(ext.__file__)
    fn = lib.ad_adam_fused_noalloc
    fn.restype = ctypes.c_int
    fn.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int64,
                   ctypes.c_int64, ctypes.c_float, ctypes.c_float, ctypes.c_float, ctypes.c_float,
                   ctypes.c_float, ctypes.c_float, ctypes.c_int, ctypes.c_void_p, ctypes.c_void_p]
    msg = lib.ad_adam_fused_noalloc_message
    msg.restype = ctypes.c_char_p
    msg.argtypes = [ctypes.c_int]
    return ext, fn, msg


def _call(fn, p, g, m, v, norm, step, blocks=0, max_norm=.5):
    stream = torch.cuda.current_stream().cuda_stream
    return fn(p.data_ptr(), g.data_ptr(), m.data_ptr(), v.data_ptr(), p.numel(), step, 3e-4, .9, .999, 1e-5,
              0., max_norm, blocks, norm.data_ptr(), stream)


def test_noalloc_matches_existing_entry_point_twice():
    ext, fn, msg = _lib()
    torch.manual_seed(0)
    n = 100_003
    p_ref = torch.randn(n, device="cuda")
    m_ref = torch.zeros(n, device="cuda")
    v_ref = torch.zeros(n, device="cuda")
    p_new, m_new, v_new = p_ref.clone(), m_ref.clone(), v_ref.clone()
    partial = torch.zeros(int(ext.ADAM_NORM_BLOCKS), device="cuda")
    norm_ref = torch.zeros(1, device="cuda")
    norm_new = torch.zeros(1, device="cuda")
    for step in (1, 2):
        g = torch.randn(n, device="cuda") * (3. if step == 1 else .01)  # clipped, then unclipped
        ext.adam_fused(p_ref, g, m_ref, v_ref, partial, norm_ref, step, 3e-4, .9, .999, 1e-5, 0., .5)
        status = _call(fn, p_new, g, m_new, v_new, norm_new, step)
        assert status == 0, msg(status)
        torch.cuda.synchronize()
        assert torch.allclose(norm_new, norm_ref, rtol=1e-5, atol=1e-5)
        for a, b in ((p_new, p_ref), (m_new, m_ref), (v_new, v_ref)):
            assert torch.allclose(a, b, rtol=1e-5, atol=1e-6)


def test_noalloc_matches_torch_adam_and_clip_in_fp32():
    """Two consecutive calls against the plain PyTorch fp32 update:
    clip_grad_norm_(0.5) then torch.optim.Adam (lr 3e-4, betas .9/.999,
    eps 1e-5)."""
    _, fn, msg = _lib()
    torch.manual_seed(1)
    n = 65_537
    ref = torch.nn.Parameter(torch.randn(n, device="cuda"))
    opt = torch.optim.Adam([ref], lr=3e-4, betas=(.9, .999), eps=1e-5, foreach=False, fused=False)
    p = ref.detach().clone()
    m, v = torch.zeros(n, device="cuda"), torch.zeros(n, device="cuda")
    norm = torch.zeros(1, device="cuda")
    for step in (1, 2):
        g = torch.randn(n, device="cuda") * (2. if step == 1 else .001)  # clipped, then unclipped
        ref.grad = g.clone()
        total = torch.nn.utils.clip_grad_norm_([ref], .5)
        opt.step()
        status = _call(fn, p, g, m, v, norm, step)
        assert status == 0, msg(status)
        torch.cuda.synchronize()
        assert torch.allclose(norm, total.reshape(1), rtol=1e-5, atol=1e-6)
        assert torch.allclose(p, ref.detach(), rtol=1e-5, atol=1e-6)
        state = opt.state[ref]
        assert torch.allclose(m, state["exp_avg"], rtol=1e-5, atol=1e-7)
        assert torch.allclose(v, state["exp_avg_sq"], rtol=1e-5, atol=1e-9)


def test_noalloc_rejects_block_count_beyond_scratch():
    _, fn, msg = _lib()
    n = 1024
    p = torch.randn(n, device="cuda")
    before = p.clone()
    g, m, v = torch.randn(n, device="cuda"), torch.zeros(n, device="cuda"), torch.zeros(n, device="cuda")
    norm = torch.zeros(1, device="cuda")
    status = _call(fn, p, g, m, v, norm, 1, blocks=1025)
    assert status == 2
    assert b"1024" in msg(status)
    torch.cuda.synchronize()
    assert torch.equal(p, before)
