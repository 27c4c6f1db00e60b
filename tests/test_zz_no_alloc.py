"""qw_quantized_matmul_argmax_static (the workspace-free logits head) against
the existing qw_quantized_matmul entry point, through the C ABI.

Collected last on purpose: it must pass both in a fresh process and after the
other GPU tests.  Tolerance as in the quantized_matmul parity tests:
|y_static - y| <= 1e-2 * max|y| + 1e-3 elementwise; the returned argmax must
be the first index of the largest logit of the returned row (exact), and that
logit must be within the same tolerance of the existing entry point's row
maximum.  Each case is run twice in a row with different activations, so a
stale maximum left in the static scratch would show.
"""
import numpy as np
import pytest

from oracle import numerics as nm
from oracle import synth

pytestmark = pytest.mark.gpu


def _dev(a, torch):
    return torch.from_numpy(a).to("cuda:0")


def _bf16_to_f32(t):
    return nm.bf16_bits_to_f32(t.cpu().numpy().view(np.uint16))


@pytest.mark.parametrize("M,K,N", [(1, 2560, 151936), (5, 2560, 151936), (8, 1024, 151936), (3, 192, 1000)])
def test_static_argmax_matches_quantized_matmul(M, K, N):
    import torch
    import qwen3_b200 as q
    w, s, b = synth.quantized_weight_c(77, 2, N, K)
    wt, st, bt = _dev(w.view(np.int32), torch), _dev(s.view(np.int16), torch), _dev(b.view(np.int16), torch)
    stream = torch.cuda.current_stream().cuda_stream
    for call in range(2):
        rng = np.random.default_rng(500 + 10 * call + M)
        x = nm.bf16_round(rng.standard_normal((M, K)).astype(np.float32))
        xt = _dev(nm.f32_to_bf16_bits(x).view(np.int16), torch)
        y_ref = torch.zeros((M, N), dtype=torch.int16, device="cuda:0")
        y_new = torch.zeros((M, N), dtype=torch.int16, device="cuda:0")
        am = torch.full((M,), -1, dtype=torch.int32, device="cuda:0")
        am_noy = torch.full((M,), -1, dtype=torch.int32, device="cuda:0")
        q.quantized_matmul(xt.data_ptr(), wt.data_ptr(), st.data_ptr(), bt.data_ptr(), y_ref.data_ptr(), M, N, K,
                           stream=stream)
        q.quantized_matmul_argmax_static(xt.data_ptr(), wt.data_ptr(), st.data_ptr(), bt.data_ptr(),
                                         y_new.data_ptr(), am.data_ptr(), M, N, K, stream=stream)
        q.quantized_matmul_argmax_static(xt.data_ptr(), wt.data_ptr(), st.data_ptr(), bt.data_ptr(), 0,
                                         am_noy.data_ptr(), M, N, K, stream=stream)
        torch.cuda.synchronize()
        yr, yn = _bf16_to_f32(y_ref), _bf16_to_f32(y_new)
        tol = 1e-2 * np.abs(yr).max() + 1e-3
        assert np.abs(yn - yr).max() <= tol, (call, np.abs(yn - yr).max(), tol)
        a, a2 = am.cpu().numpy(), am_noy.cpu().numpy()
        assert list(a) == list(np.argmax(yn, axis=1)), (call, a, np.argmax(yn, axis=1))
        assert list(a2) == list(a), (call, a2, a)
        for m in range(M):
            assert yr[m, a[m]] >= yr[m].max() - tol, (call, m)


def test_static_argmax_rejects_oversize():
    import torch
    import qwen3_b200 as q
    M, K = 8, 64
    N = 16 * (q.STATIC_AMAX_SLOTS // M) + 16  # one row block more than the scratch holds
    dummy = torch.zeros(16, dtype=torch.int32, device="cuda:0")
    p = dummy.data_ptr()
    with pytest.raises(q.Error, match="exceeds the static scratch"):
        q.quantized_matmul_argmax_static(p, p, p, p, 0, p, M, N, K)
    with pytest.raises(q.Error):
        q.quantized_matmul_argmax_static(p, p, p, p, 0, p, 9, 16, K)
    # a row too long for the GEMV's shared-memory staging is an argument error naming the sizes
    with pytest.raises(q.Error, match="does not fit"):
        q.quantized_matmul_argmax_static(p, p, p, p, 0, p, 8, 16, 25600)


def test_static_argmax_on_two_devices():
    """The scratch address and the kernel's shared-memory opt-in are per device:
    a call on device 1 after device 0 in the same process must work."""
    import torch
    import qwen3_b200 as q
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    M, K, N = 8, 2560, 4096
    w, s, b = synth.quantized_weight_c(78, 3, N, K)
    rng = np.random.default_rng(9)
    x = nm.f32_to_bf16_bits(nm.bf16_round(rng.standard_normal((M, K)).astype(np.float32))).view(np.int16)
    got = []
    for dev in (0, 1):
        d = f"cuda:{dev}"
        with torch.cuda.device(dev):
            wt, st_, bt = (torch.from_numpy(a).to(d) for a in (w.view(np.int32), s.view(np.int16), b.view(np.int16)))
            xt = torch.from_numpy(x).to(d)
            am = torch.full((M,), -1, dtype=torch.int32, device=d)
            q.quantized_matmul_argmax_static(xt.data_ptr(), wt.data_ptr(), st_.data_ptr(), bt.data_ptr(), 0,
                                             am.data_ptr(), M, N, K, stream=torch.cuda.current_stream(dev).cuda_stream)
            torch.cuda.synchronize(dev)
            got.append(am.cpu().numpy())
    assert list(got[0]) == list(got[1])
