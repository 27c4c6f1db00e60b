// Per-element output treatment shared by the quantized matmul kernels
// (qmatmul.cu: qgemv / qgemm, qgemm_tc.cu: the tcgen05 prefill GEMM), so every
// path rounds and combines identically.
#pragma once
#include "kernels.h"

namespace qw {

// Final per-element epilogue (every mode except EPI_LOGITS).
QW_DEV void store_out(const QmmArgs& a, int si, int epi, int row, int feat, int col, float v0, float v1) {
    if (epi == EPI_SWIGLU) {
        const float g = bfr(v0), u = bfr(v1);
        const float sg = bfr(1.0f / (1.0f + expf(-g)));
        const float act = bfr(__fmul_rn(g, sg));
        bf16* y = reinterpret_cast<bf16*>(a.seg[0].y);
        y[(size_t)col * a.seg[0].ldy + feat] = f2bf(__fmul_rn(act, u));
        return;
    }
    const QSeg& sg = a.seg[si];
    const size_t idx = (size_t)col * sg.ldy + row;
    if (epi == EPI_F32) {
        reinterpret_cast<float*>(sg.y)[idx] = v0;
    } else if (epi == EPI_F32_PUSH) {
        // this rank's partial into every rank's receive slot (peer stores over NVLink)
        const TpPush& p = a.push;
        const unsigned e = *p.epoch + 1u;
        const size_t off = ((size_t)((e & 1u) * p.n + p.self) * TP_PUSH_ROWS + col) * p.H + row;
        for (int q = 0; q < p.n; ++q) p.recv[q][off] = v0;
    } else if (epi == EPI_RESID) {
        bf16* y = reinterpret_cast<bf16*>(sg.y);
        y[idx] = f2bf(__fadd_rn(bf2f(y[idx]), bfr(v0)));
    } else {
        reinterpret_cast<bf16*>(sg.y)[idx] = f2bf(v0);
    }
}

}  // namespace qw
