// Host-side launchers of the kokoro-b200 kernels (one per kernel family). Every launcher
// enqueues on the given stream and returns the launch status.
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>
#include "kk_common.cuh"

namespace kk {

// Per-item table of a batch: token rows [tok_start, tok_start + tok_len) and frame span
// [a, a + n) of the N domain (src/gpu_batch.rs:189-263).
struct ItemTab {
  int tok_start, tok_len, a, n;
};

// ---- convolution / linear
cudaError_t launch_conv_simt(const ConvArgs& a, cudaStream_t st);
size_t conv_simt_smem(const ConvArgs& a);

// ---- token side
// ALBERT embeddings: word[id] + token_type[0] + pos[i] -> LayerNorm(eps 1e-12) (src/albert.rs:67-81)
cudaError_t launch_albert_embed(const int* ids, const int* row_item, const ItemTab* items, int rows,
                                const float* word, const float* pos, const float* tt0, const float* g,
                                const float* b, float* out, cudaStream_t st);
// out[r, 0:d] = src[tab[r], 0:d] (tab < 0 -> 0); tab == null: identity row index with row_item mask
cudaError_t launch_gather_rows(const float* src, int lds, const int* tab, int rows, int d, float* out,
                               int ldo, cudaStream_t st);
// y[t, 0:cout] = bias + W x[t] for K = 1 layers with cout <= 4 (the F0 / N projections), one warp
// per row; x gap rows (IN_MASK) give the bias alone
bool rowproj_supported(const ConvArgs& a);
cudaError_t launch_rowproj(const ConvArgs& a, cudaStream_t st);
// text embedding rows (gap rows -> 0)
cudaError_t launch_embed_rows(const int* ids, const int* row_item, int rows, const float* table, int d,
                              float* out, cudaStream_t st);
// Row LayerNorm with f64 reductions (kernels/kokoro.cu:44-82).
//  mode 0: affine; mode 1: affine + leaky(slope);
//  mode 2: AdaLayerNorm (no affine, (1 + g) * x + b with gb rows per item, kernels/kokoro.cu:337-372),
//          written to y[:, 0:d], followed by the item's style in y[:, d:d+sdim] (cat_style_rows_seg,
//          :375-383); gap rows of y -> 0.
// ypre (optional, d = 512 / 768, modes 0 / 1): the output rows also as bf16 window planes (the
// IN_PRE operand layout of kk_common.cuh, ypre_rows rows per plane) for a following tensor-core layer.
cudaError_t launch_ln_rows(const float* x, int ldx, int rows, int d, const float* g, const float* b,
                           float eps, int mode, float slope, const int* row_item, const float* gb,
                           int ldgb, const float* style, int sdim, float* y, int ldy, cudaStream_t st,
                           void* ypre = nullptr, long ypre_rows = 0);
// cat_style_rows_seg: y[:, d:d+sdim] = style[item]; gap rows of y[:, 0:d+sdim] -> 0
cudaError_t launch_cat_style(const int* row_item, int rows, int d, const float* style, int sdim, float* y,
                             int ldy, cudaStream_t st);
// Per-item multi-head attention over token rows, fp32 online softmax (src/gpu_batch.rs:429-442).
cudaError_t launch_attention_f32(const float* qkv, int ldqkv, const ItemTab* items, int B, int max_len,
                                 float* ctx, int ldc, cudaStream_t st);
// The same attention on tcgen05 tensor cores (bf16 Q, K, V and P, fp32 accumulation and softmax).
// work: (item, first query row) per 128-query tile, grouped by item length into the buckets
// T <= 128, T <= 256 and T <= 512 of n_work[0..2] entries. err receives 3 if an MMA wait expires.
// With ctx_pre set, ctx is written only as bf16 window planes (IN_PRE layout, ctx_pre_rows rows per
// plane; head h = 64-channel block h) for the output projection, and ctx is not touched.
// qkv_bf16: the qkv rows are bf16 (ldqkv elements apart, a multiple of 8), else f32.
cudaError_t launch_attention_tc(const void* qkv, int ldqkv, bool qkv_bf16, const ItemTab* items, const int2* work,
                                const int n_work[3], float* ctx, int ldc, int* err, cudaStream_t st,
                                void* ctx_pre = nullptr, long ctx_pre_rows = 0);

// ---- LSTM recurrence (one launch per BiLSTM, thread-block clusters; kk_lstm.cu)
// Items sorted longest-first form G groups of LSTM_IPG; one cluster of 8 CTAs runs each
// (group, direction).
struct LstmArgs {
  const float* gx;    // [rows][ldgx]: dir d gate g unit j at column d*4H + g*H + j (includes b_ih)
  int ldgx;
  const float* whh;   // [2][4H][H]
  const float* bhh;   // [2][4H]
  float* out;         // [rows][ldo]: dir d unit j at column d*H + j
  int ldo;
  const int* gstart;  // [G][IPG] first row of each group member, longest first (unused slots 0)
  const int* glen;    // [G][IPG] its length (unused slots 0)
  const int* gact;    // [G][Tmax] members of group g still running at step s
  int G, IPG, Tmax;
  int tc;             // 1: tcgen05 recurrence (BF16 mode: bf16 hi/lo split operands, fp32 accumulation)
  int* err;           // tc: set to 4 if an MMA completion wait expires
};
constexpr int LSTM_IPG = 32;
cudaError_t launch_lstm(const LstmArgs& a, cudaStream_t st);

// ---- AdaIN statistics: per (item, channel) mean / rstd over the item's span (biased variance,
// eps 1e-5; shifted f32 partial sums combined in f64, kernels/kokoro.cu:776-810)
cudaError_t launch_stats(const float* x, int ldx, int C, const ItemTab* items, int B, int scale,
                         int plus1, int max_len, double* part, float* mean, float* rstd,
                         cudaStream_t st);

// mean / rstd from fused output sums (tensor-core conv epilogue): part[b][c] = (sum, sum of squares)
// over the item's span of the domain (scale, plus1); biased variance, eps 1e-5.
cudaError_t launch_stats_from_sums(const double* part, int C, const ItemTab* items, int B, int scale, int plus1,
                                   float* mean, float* rstd, cudaStream_t st);

// AdaIN folded into one affine map per (item, channel) for the bf16 tensor-core path:
// coef[b][c] = (A, B) with AdaIN(x) = x * A + B, A = (1 + gamma) * rstd * nw,
// B = (1 + gamma) * (nb - mean * rstd * nw) + beta.
cudaError_t launch_adain_coef(const float* mean, const float* rstd, const float* nw, const float* nb,
                              const float* gb, int ldgb, int B, int C, float2* coef, cudaStream_t st);

// The input transform of a convolution (a.in_mode over a.x, a.in_up2, a.din, AdaIN coef / alpha)
// applied once, written as bf16 window planes for IN_PRE (layout in ConvArgs::xpre): pre_rows =
// PRE_PAD_FRONT + a.L_in + PRE_PAD_BACK, planes = 8 * ceil(cin / 64); pad rows and channels past
// cin are zero.
cudaError_t launch_prologue_bf16(const ConvArgs& a, void* xpre, long pre_rows, cudaStream_t st);

// AdaIN + leaky ReLU (0.2) followed by the depthwise ConvTranspose1d(k3, s2, p1, op1) "pool"
// (adain_apply_seg + dw_convT_k3s2, kernels/kokoro.cu:152-167, 317-334): x [L][C] -> y [2L][ldy]
cudaError_t launch_adain_pool(const float* x, int C, int L, const ConvArgs& pro, const float* pw,
                              const float* pb, float* y, int ldy, cudaStream_t st);

// durations_from_logits (src/model.rs:90-99) per token row: dur = max(1, rne(sum sigmoid / speed))
cudaError_t launch_durations(const float* logits, int ldl, const int* row_item, const float* speed,
                             int rows, int* dur, float* q, cudaStream_t st);

// F0_conv / N_conv (Conv1d 1->1, k3, s2, p1) on the masked 2N curves, written into up to three
// column destinations of N-domain buffers.
struct CurveConv {
  const float* w;   // [3]
  float b;
};
cudaError_t launch_curve_conv(const float* f0, const float* nc, Dom d2, int LN, CurveConv wf, CurveConv wn,
                              float* dst0, int ld0, int col0, float* dst1, int ld1, int col1,
                              float* dst2, int ld2, int col2, cudaStream_t st);

// ---- harmonic source, STFT, iSTFT (kernels/kokoro.cu:188-302, 470-508)
cudaError_t launch_sine_phase(const float* f0, int L2, const ItemTab* items, int B, float* pp,
                              cudaStream_t st);
cudaError_t launch_har_source(const float* f0, const float* pp, int L2, const ItemTab* items,
                              const int* col_item_n, int LN, const uint64_t* seeds, const float* noise,
                              const long long* noise_off, const float* lw, float lb, float* har,
                              cudaStream_t st);
cudaError_t launch_stft(const float* har, const ItemTab* items, Dom d120, float* spec, int lds,
                        cudaStream_t st);
cudaError_t launch_istft(const float* post, int ldp, const ItemTab* items, Dom d120, const int* col_item_n,
                         int LN, float* audio, cudaStream_t st);

// ---- glue
// y = ((r0 + r1) + r2) / 3 over n elements
cudaError_t launch_sum3(const float* r0, const float* r1, const float* r2, float* y, long n, cudaStream_t st);
// stage-1 reflection pad (1, 0) per item plus the noise branch: x[o] = pad(y)[o] + xs[o]
cudaError_t launch_reflect_add(const float* y, const float* xs, int C, const ItemTab* items, Dom d120,
                               float* x, cudaStream_t st);
// the same for C = 128, adding the result's per-(item, channel) sum and sum of squares into part
// (f64 [B][128][2], zeroed by the caller): the AdaIN statistics of the stage-1 input (BF16 mode)
cudaError_t launch_reflect_add_stats(const float* y, const float* xs, const ItemTab* items, Dom d120, float* x,
                                     double* part, cudaStream_t st);
// PCM_16 conversion of n samples (600 per N-domain column) with per-item clip counts (pre-zeroed)
cudaError_t launch_pcm16(const float* audio, long n, const int* col_item_n, int16_t* out, unsigned long long* clipped,
                         cudaStream_t st);
// dst[r, c0d + j] = src[r, c0s + j] for j < ncol
cudaError_t launch_copy_cols(const float* src, int lds, int c0s, float* dst, int ldd, int c0d, int rows,
                             int ncol, cudaStream_t st);

// Bounded-wait self-test: one thread waits, with the pipelines' bounded mbarrier wait and a limit of
// limit_ns, on a barrier nothing arrives on; the wait expires and sets *err (code 2).
cudaError_t launch_wait_selftest(int* err, unsigned long long limit_ns, cudaStream_t st);

// f64 twiddles [cos 11x20 | sin 11x20] and the periodic Hann window (src/gpu.rs:93-103)
cudaError_t upload_stft_constants(cudaStream_t st);

}  // namespace kk
