"""quantized_matmul parity: CUDA (qgemv M<=8 / qgemm M>8) vs the CPU oracle.

Shapes are benchmark config 2 (Qwen3-4B projections) plus odd-sized edge cases.
Tolerance: the CUDA path and the oracle both accumulate in fp32 and round the
output once to bf16, so they agree to within one bf16 rounding of values of
the output's magnitude: |gpu - ref| <= 1e-2 * max|ref| + 1e-3 elementwise, and
at least 99% of elements bit-identical.
"""
import numpy as np
import pytest

from oracle import numerics as nm

pytestmark = pytest.mark.gpu

SHAPES_4B = [(2560, 4096), (2560, 1024), (4096, 2560), (2560, 9728), (9728, 2560)]


def _case(M, K, N, seed):
    rng = np.random.default_rng(seed)
    w, s, b = nm.quantized_weight(seed, 99, N, K)
    x = nm.bf16_round(rng.standard_normal((M, K)).astype(np.float32))
    return x, w, s, b


def _run_gpu(x, w, s, b):
    import torch
    import qwen3_b200 as q
    dev = torch.device("cuda:0")
    M, K = x.shape
    N = w.shape[0]
    xt = torch.from_numpy(nm.f32_to_bf16_bits(x).view(np.int16)).to(dev)
    wt = torch.from_numpy(w.view(np.int32)).to(dev)
    st = torch.from_numpy(s.view(np.int16)).to(dev)
    bt = torch.from_numpy(b.view(np.int16)).to(dev)
    yt = torch.zeros((M, N), dtype=torch.int16, device=dev)
    q.quantized_matmul(xt.data_ptr(), wt.data_ptr(), st.data_ptr(), bt.data_ptr(), yt.data_ptr(), M, N, K,
                       stream=torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    return nm.bf16_bits_to_f32(yt.cpu().numpy().view(np.uint16))


def _check(y, ref):
    tol = 1e-2 * np.abs(ref).max() + 1e-3
    err = np.abs(y - ref)
    assert err.max() <= tol, f"max err {err.max()} > {tol}"
    assert (y == ref).mean() >= 0.99, f"only {(y == ref).mean():.4f} bit-identical"


@pytest.mark.parametrize("M", [1, 5, 128])
@pytest.mark.parametrize("K,N", SHAPES_4B)
def test_qmatmul_4b_shapes(M, K, N):
    x, w, s, b = _case(M, K, N, seed=1000 + K + N)
    ref = nm.bf16_round(x @ nm.dequantize(w, s, b).T)
    _check(_run_gpu(x, w, s, b), ref)


@pytest.mark.parametrize("M,K,N", [(1, 64, 16), (3, 192, 40), (8, 320, 96), (9, 128, 48), (33, 256, 200),
                                   (2048, 2560, 1024),
                                   # warp-ring GEMV (>= one 16-row tile per SM, K a multiple of 512): ragged
                                   # last tile, one-granule tiles with most warps idle, tiles split over many
                                   # warps, eight columns
                                   (3, 1024, 4741), (1, 512, 2400), (2, 4096, 2371), (8, 1536, 2376),
                                   # long rows: 4 warps per CTA (8 columns of 9728 staged inputs)
                                   (8, 9728, 2560)])
def test_qmatmul_edges(M, K, N):
    x, w, s, b = _case(M, K, N, seed=7 + M + K + N)
    ref = nm.bf16_round(x @ nm.dequantize(w, s, b).T)
    _check(_run_gpu(x, w, s, b), ref)


def test_qmatmul_lm_head_m1():
    x, w, s, b = _case(1, 2560, 151936, seed=5)
    ref = nm.bf16_round(x @ nm.dequantize(w, s, b).T)
    _check(_run_gpu(x, w, s, b), ref)


@pytest.mark.parametrize("bn", ["128", "256"])
@pytest.mark.parametrize("M,K,N", [(300, 1024, 384), (513, 2560, 200)])
def test_qmatmul_tc_tile_widths(bn, M, K, N, monkeypatch):
    """Both activation tile widths of the tcgen05 prefill GEMM (ragged M and N)."""
    monkeypatch.setenv("QW_TC_BN", bn)
    x, w, s, b = _case(M, K, N, seed=31 + M + N)
    ref = nm.bf16_round(x @ nm.dequantize(w, s, b).T)
    _check(_run_gpu(x, w, s, b), ref)


@pytest.mark.parametrize("M", [1, 5, 8])
def test_qmatmul_long_rows_32b_down_proj(M):
    """Qwen3-32B down_proj rows (K = 25600): the GEMV's whole-K weight slab does
    not fit in shared memory, so rows of M <= 8 take the tiled GEMM instead."""
    x, w, s, b = _case(M, 25600, 160, seed=61 + M)
    ref = nm.bf16_round(x @ nm.dequantize(w, s, b).T)
    _check(_run_gpu(x, w, s, b), ref)


@pytest.mark.parametrize("M,K,N", [(1, 2560, 6144), (5, 9728, 2560), (1, 2560, 151936)])
def test_qmatmul_inputs_written_by_previous_kernel(M, K, N):
    """The standalone op starts while the previous kernel drains (programmatic
    launch); weights, scales, biases and x written by that kernel must still be
    the ones it reads.  Each call's operands are produced by a device copy
    launched directly before it on the same stream, into buffers that held
    other values, and consecutive calls write the same output."""
    import torch
    import qwen3_b200 as q
    dev = torch.device("cuda:0")
    cases = [_case(M, K, N, seed=400 + i) for i in range(3)]
    srcs = [tuple(torch.from_numpy(a.view(dt)).to(dev) for a, dt in
                  zip((nm.f32_to_bf16_bits(x), w, s, b), (np.int16, np.int32, np.int16, np.int16)))
            for (x, w, s, b) in cases]
    bufs = [torch.empty_like(t) for t in srcs[0]]
    yt = torch.zeros((M, N), dtype=torch.int16, device=dev)
    outs = []
    stream = torch.cuda.current_stream()
    for i in range(3):
        # the weight words last: the kernel directly before the matmul writes them
        for j in (0, 2, 3, 1):
            bufs[j].copy_(srcs[i][j], non_blocking=True)
        q.quantized_matmul(bufs[0].data_ptr(), bufs[1].data_ptr(), bufs[2].data_ptr(), bufs[3].data_ptr(),
                           yt.data_ptr(), M, N, K, stream=stream.cuda_stream)
        outs.append(yt.clone())
    torch.cuda.synchronize()
    for (x, w, s, b), yo in zip(cases, outs):
        ref = nm.bf16_round(x @ nm.dequantize(w, s, b).T)
        _check(nm.bf16_bits_to_f32(yo.cpu().numpy().view(np.uint16)), ref)
