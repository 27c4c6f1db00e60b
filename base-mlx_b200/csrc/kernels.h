// Kernel launch interface shared by the runtime (host) and the .cu kernel files.
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

#include "common.cuh"

namespace qw {

// Output treatment of a quantized matmul.
enum Epi : int {
    EPI_STORE = 0,   // y = bf16(acc)
    EPI_RESID = 1,   // y = bf16(y + bf16(acc))             (o_proj / down_proj + residual)
    EPI_SWIGLU = 2,  // y = bf16(bf16(g*bf16(sigmoid(g))) * u), g/u = bf16(gate/up acc)
    EPI_LOGITS = 3,  // bf16 logits (optional store) + fused argmax per row
    EPI_F32 = 4,     // y_f32 = acc (tensor-parallel partial sums)
    EPI_F32_PUSH = 5,  // tensor parallel, decode: acc stored into every rank's receive slot (TpPush)
};

// One quantized linear segment [n rows x K] (MLX layout).
struct QSeg {
    const uint32_t* w;  // [n, K/8]
    const bf16* s;      // [n, K/64]
    const bf16* b;      // [n, K/64]
    void* y;            // output base (bf16 or fp32), element (m, row) at y[m*ldy + row]
    int n;
    int ldy;
    int rb0;            // first row block of this segment in the launch grid
};

// Tensor-parallel reduction over peer memory (decode rows <= TP_PUSH_ROWS): a
// GEMV with EPI_F32_PUSH writes its fp32 partial of output (row m, feature f)
// into every rank q's exchange block, recv[q][((e & 1) * n + self) *
// TP_PUSH_ROWS + m][f] (e = *epoch + 1, the reduction's epoch); each CTA then
// arrives on a local counter (acquire-release, GPU scope) and the last one
// stores e into every rank's flag for this source rank with a system-scope
// release (the arrivals chain every CTA's stores before it).
constexpr int TP_PUSH_MAX = 8;   // ranks
constexpr int TP_PUSH_ROWS = 8;  // rows per reduction
struct TpPush {
    float* recv[TP_PUSH_MAX];     // each rank's receive region (this rank's own at [self])
    unsigned* flag[TP_PUSH_MAX];  // each rank's flag for this source rank
    const unsigned* epoch;        // this rank's completed reductions
    unsigned* ctr;                // CTA arrivals of the GEMV (zero between launches)
    int n, self, H;
};

struct QmmArgs {
    const bf16* x;   // [M, ldx] activations
    int ldx;
    int M, K;
    const bf16* norm_w;  // optional RMSNorm weight [K] applied to x first (decode path)
    float eps;
    QSeg seg[3];
    int nseg;
    int epi;
    int nrb;             // row blocks in the grid (gridDim.x)
    // fused argmax (EPI_LOGITS): per-CTA (logit, index) maxima, reduced by
    // launch_amax_finalize
    unsigned long long* amax_partial;  // [nrb, M]
    int store_logits;
    int amax_row_offset;               // global index of row 0 (vocab-parallel shards)
    int* err;
    TpPush push;                       // EPI_F32_PUSH
    // 0: the weights are static (model weights), so the GEMV copies them into
    // shared memory before the programmatic-launch wait.  1: the previous
    // kernel on the stream may have written them (the standalone op), so only
    // L2 prefetch hints run before the wait and the copies after it.
    int weights_after_wait;
    // tcgen05 GEMM split over K (launch_qgemm_tc sets both): > 1 -> CTA z of
    // gridDim.z covers whole 8-group chunks [z C / ksplit, (z + 1) C / ksplit)
    // of the C = K / 512 chunks and stores fp32 partials kpart[z][col][row];
    // a reduce kernel sums them in z order and applies the epilogue
    int ksplit;
    float* kpart;
};

// Decode / verify path: M <= 8.
cudaError_t launch_qgemv(QmmArgs a, cudaStream_t st, bool pdl, int num_sms);
// Row blocks of the qgemv grid for these segments (size of amax_partial / M).
int qgemv_row_blocks(const QmmArgs& a);
// Whether the GEMV's whole-K weight slab (16 or 32 rows x K) fits in shared
// memory; long rows that do not (K = 25600 at 220 KB) go to the tiled GEMM.
bool qgemv_fits(const QmmArgs& a);
// Largest K (a multiple of 64) whose single-segment GEMV fits, at M rows.
int qgemv_max_k(int M);
// argmax[m] (and optionally packed keys) from the EPI_LOGITS per-CTA maxima.
cudaError_t launch_amax_finalize(const unsigned long long* partial, int nrb, int M, int* out,
                                 unsigned long long* keys_out, cudaStream_t st);
// Prefill path: M > 8 (no norm prologue, no argmax; EPI_STORE/RESID/SWIGLU/F32).
cudaError_t launch_qgemm(QmmArgs a, cudaStream_t st, int num_sms);
// Prefill path on the tcgen05 tensor cores (qgemm_tc.cu): M > 8, K a multiple
// of 128, no norm prologue, no argmax.  `scratch` holds the fp16 copy of x
// (qgemm_tc_scratch_bytes).  Callers fall back to launch_qgemm when
// qgemm_tc_supported is false.
bool qgemm_tc_supported(const QmmArgs& a);
size_t qgemm_tc_scratch_bytes(int M, int K);
// K split the standalone op gives a launch whose output tiles leave SMs idle
// (one segment, plain / fp32 / residual store; 1: no split), and the scratch
// it needs beyond qgemm_tc_scratch_bytes for the fp32 partials.
int qgemm_tc_ksplit(const QmmArgs& a, int num_sms);
size_t qgemm_tc_ksplit_bytes(const QmmArgs& a, int ksplit);
cudaError_t launch_qgemm_tc(QmmArgs a, void* scratch, size_t scratch_bytes, cudaStream_t st, int ksplit = 1);

// ---- other kernels ------------------------------------------------------
struct AttnArgs {
    const bf16* q; const bf16* k; const bf16* v;   // [S, ldq] etc.
    int ldq, ldk, ldv;
    const bf16* q_norm_w; const bf16* k_norm_w; float eps;
    const float* rope_cos; const float* rope_sin;  // [max_pos, 64]
    bf16* kcache; bf16* vcache;                    // this layer: [Hkv, max_pos, 128]
    int max_pos;
    const int* seq_len;                            // device offset (positions already cached)
    int S, Hq, Hkv;                                // local heads
    float scale;
    float* part;          // [Hkv, nsplit, R, 130]
    unsigned* counters;   // merge counters: [Hq] (split attention: kvh * G + first query head of the item; the kernel-chain attention uses [Hkv])
    bf16* out; int ldo;   // [S, Hq*128]
    int nsplit;
    int* err;
    unsigned long long* prof;  // persistent kernel diagnostics: this item's timing stamps, or null
};
cudaError_t launch_attn_decode(const AttnArgs& a, cudaStream_t st, bool pdl);
// prefill: q/k norm + rope + cache write for all S rows, roped q to qout
cudaError_t launch_qk_norm_rope_kvwrite(const AttnArgs& a, bf16* qout, cudaStream_t st);
cudaError_t launch_attn_prefill(const AttnArgs& a, const bf16* qroped, cudaStream_t st);

cudaError_t launch_embed(const int* ids, int S, const uint32_t* w, const bf16* s, const bf16* b,
                         int H, int vocab, bf16* x, int* err, cudaStream_t st, bool pdl);
cudaError_t launch_rmsnorm(const bf16* x, const bf16* w, bf16* y, int S, int H, float eps,
                           cudaStream_t st);
cudaError_t launch_argmax_rows(const bf16* logits, int rows, int V, int* out, unsigned long long* keys_out,
                               int index_offset, cudaStream_t st);
cudaError_t launch_keys_to_index(const unsigned long long* keys, int n, int* out, cudaStream_t st);
cudaError_t launch_resid_add_f32(bf16* x, const float* p, int n, cudaStream_t st);

// Random-init: fill a quantized tensor [rows, K] (rows r0.. of a [*, Kfull] tensor,
// columns k0.. of it) from the seeded generator.
cudaError_t launch_init_qweight(uint32_t* w, bf16* s, bf16* b, int rows, int K, int row0, int k0,
                                int Kfull, uint64_t key, float mult, cudaStream_t st);
cudaError_t launch_init_norm(bf16* w, int n, uint64_t key, float mult, int ones, cudaStream_t st);

// ---- step control (device-side generation loops) ----------------------
struct StepCtl {
    int produced;    // tokens picked so far (includes a terminating EOS)
    int n_out;       // tokens written to out
    int done;        // 1 once EOS or max_new reached
    int finish;      // 0 length, 1 stop
    int max_new;
    int n_eos;
    int eos[8];
};
// Batched greedy decode control block (device): the step count, each
// sequence's output count and whether it stopped at EOS; `done` once every
// sequence stopped or the token budget is spent (later replays do nothing).
struct BatchCtl {
    int produced;  // tokens picked per sequence so far (the prefill's included)
    int max_new;
    int done;
    int n_eos;
    int eos[8];
    int n_out[8];
    int stopped[8];
};
// Temperature / top-p sampling parameters (SamplingParams fields that
// engine.rs:195-263 pick_next reads).  seed drives a counter-based draw:
// u = top 24 bits of splitmix64(seed ^ splitmix64(counter)) / 2^24, counter =
// tokens already picked, or 0 for every token when same_draw != 0 (the
// reference re-seeds its generator from the same seed at every token).
constexpr size_t QW_SAMPLE_CTRL_BYTES = 16384;  // sampling control block (grid barrier, partials, histograms)
struct SampleCfg {
    float temperature;
    float top_p;
    unsigned long long seed;
    int same_draw;
};
struct SampleArgs {
    const bf16* logits;        // [V] bf16 (row of the last position)
    int V;
    const SampleCfg* cfg_dev;  // device copy (generation loop), else `cfg`
    SampleCfg cfg;
    float* probs;              // scratch [V]
    StepCtl* ctl;              // generation loop bookkeeping, or null (standalone)
    int* next_tok;
    int* out;
    unsigned long long counter;  // standalone: the draw's counter
    int* token_out;              // standalone: the picked token
    void* ctrl;                  // QW_SAMPLE_CTRL_BYTES control block, zero before its first use
    int* err;                    // device error flags (timeouts), may be null
    // speculative sampling: the draw's counter = *ctr_iter * 64 + ctr_base when
    // ctr_iter is set; desc_out receives the nucleus of `probs` (which then
    // holds the row's softmax); no_draw skips the draw (token_out untouched)
    const int* ctr_iter;
    int ctr_base;
    struct SpDesc* desc_out;
    int no_draw;
    const int* gate;  // nonzero: the launch does nothing (a finished loop's replays)
};
// The top-p nucleus of a probability row p (softmax of logits / t): x is in it
// iff found == 0, or p[x] > value, or p[x] == value and x <= tie_idx (value =
// the float with bits `key`); P(x) = p[x] / renorm inside it, 0 outside.
struct SpDesc {
    uint32_t key;
    int tie_idx;
    float renorm;
    int found;
};
// softmax(logits / t), nucleus of cumulative mass >= top_p in descending-
// probability order (ties by index), categorical draw inside it: one
// cooperative grid (sample.cu).
cudaError_t launch_sample(const SampleArgs& a, cudaStream_t st);

// After a forward of S rows: seq_len += S (skipped while *gate != 0); greedy
// loop bookkeeping when ctl != null.
cudaError_t launch_step_finish(int* seq_len, int S, const int* argmax, StepCtl* ctl, int* next_tok,
                               int* out, const int* gate, cudaStream_t st, bool pdl);

}  // namespace qw
