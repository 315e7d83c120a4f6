// Shared definitions of the kokoro-b200 engine: the ragged time-major layout, the convolution
// argument block, and device helpers used by every kernel file.
//
// Layout. Every activation is time-major: row = time step (or token), channels contiguous,
// [rows][ld] with ld >= channels. Items of a batch are concatenated along time with zero gaps,
// exactly like the reference's gap-separated layout (src/gpu_batch.rs:26-59,
// docs/design/BATCHING.md): token domain gap GAP_T = 2 rows, frame (N) domain gap GAP_N = 2,
// and the derived frame domains are fixed multiples of the N domain (2N, 20N, 120N + 1, 600N
// samples), so item b always starts at scale * A_b.
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

namespace kk {

constexpr int GAP_T = 2;
constexpr int GAP_N = 2;
constexpr int STYLE = 128;
constexpr int HID = 512;

// One time domain of the ragged layout. Token domain: rows map to items through row_item.
// Frame domains: column c belongs to item col_item_n[c / scale]; with plus1, the column just
// past an item's scaled span (the 120N+1 domain's extra frame) also belongs to that item.
struct Dom {
  const int* item_tab;  // token domain: row_item [L]; frame domains: col_item_n [LN]
  int LN;               // length of the N domain (frame domains)
  int scale;            // 0 = token domain; else 1, 2, 20, 120, 600
  int plus1;            // 120N+1 domain
  int L;                // rows of this domain
};

__device__ __forceinline__ int dom_item(const Dom& d, int c) {
  if (c < 0 || c >= d.L) return -1;
  if (d.scale == 0) return d.item_tab[c];
  int q = c / d.scale;
  int b = q < d.LN ? d.item_tab[q] : -1;
  if (b >= 0) return b;
  if (d.plus1 && q >= 1 && q * d.scale == c) {
    int pb = d.item_tab[q - 1];
    if (pb >= 0) return pb;
  }
  return -1;
}

// Input transform applied while a convolution stages its input (the reference applies these as
// separate passes: mask_gaps, adain_apply_seg, and the fused AdaIN+Snake prologue of
// conv1d_wmma_bf16_snake, kernels/kokoro.cu:310-334, 660-714).
enum InMode : int {
  IN_NOMASK = 0,     // x as is (linear layers over token rows)
  IN_MASK = 1,       // x, gap rows -> 0
  IN_ADAIN_LEAKY = 2,// leaky(AdaIN(x)), gap rows -> 0
  IN_ADAIN_SNAKE = 3,// snake(AdaIN(x)), gap rows -> 0
  IN_LEAKY_MASK = 4, // leaky(x), gap rows -> 0
  IN_PRE = 5         // tensor-core path: input already transformed into bf16 window planes (xpre)
};

// Zero rows around the bf16 window planes of IN_PRE inputs: a tile's window starts at most
// (K-1)*dil/2 <= 25 rows before row 0 and ends at most 255 + (K-1)*dil rows past the last row.
constexpr int PRE_PAD_FRONT = 32;
constexpr int PRE_PAD_BACK = 320;

enum OutMode : int {
  OUT_STORE = 0,     // y = acc + bias
  OUT_ADD = 1,       // y += acc + bias
  OUT_PLUS = 2,      // y = ((acc + bias) + sc) * oscale
  OUT_GELU = 3,      // y = gelu_new(acc + bias)
  OUT_GELU_PRE = 4,  // gelu_new(acc + bias) written as bf16 window planes (ypre), the IN_PRE input of a
                     // following layer, instead of f32 rows (tensor-core path, cout a multiple of 64)
  OUT_STORE_BF = 5   // acc + bias rounded to bf16 rows (y holds __nv_bfloat16; tensor-core path, no
                     // statistics): the attention's Q / K / V, which it rounds to bf16 anyway
};

struct ConvArgs {
  // input [L_in][ldx] f32
  const float* x;
  // optional (pre-transform route only): the input row is ((x + x_b) + x_c) / 3, the mean of a
  // generator stage's three resblocks, formed while the input is transformed (same ldx)
  const float* x_b;
  const float* x_c;
  int ldx, cin, L_in;
  int in_mode;
  int in_up2;  // read row t/2 (nearest x2 upsample of the input)
  float slope;
  const float* mean;  // [B][cin]
  const float* rstd;  // [B][cin]
  const float* nw;    // [cin]
  const float* nb;    // [cin]
  const float* gb;    // gamma|beta rows: item b at gb + b*ldgb, gamma [0,cin), beta [cin,2cin)
  int ldgb;
  const float* alpha; // [cin]
  const float2* coef; // optional [B][cin] AdaIN folded to x * A + B (tensor-core path only)
  Dom din;            // domain of the input rows (after in_up2)
  // weights: f32 [K][cout][cin] (SIMT path)
  const float* w;
  const float* bias;  // [cout] or null
  int cout, K, dil, pad, stride;
  // output [L_out][ldy]
  float* y;
  int ldy, L_out;
  int out_mode;
  const float* sc;  // OUT_PLUS shortcut [L_out][ldsc]
  int ldsc;
  float oscale;
  // optional fused AdaIN statistics of the output (tensor-core path): per (item, channel)
  // sum and sum of squares, accumulated into stat[(b * cout + co) * 2 + {0, 1}] (f64, pre-zeroed)
  double* stat;
  Dom dout;           // domain of the output rows (item lookup for stat)
  // IN_PRE: bf16 planes [64-channel block][8-channel chunk][pre_rows][8], row r of the input domain
  // at plane row PRE_PAD_FRONT + r (chunk j holds channels 4j..4j+3 and 32+4j..32+4j+3)
  const void* xpre;
  long pre_rows;
  // OUT_GELU_PRE: output planes in the same layout, ypre_rows rows per plane
  void* ypre;
  long ypre_rows;
  // negative control (tests, SIMT path): gap rows of the input are read as they are instead of as
  // zeros (the reference's KOKORO_BATCH_NEGCTL_NOMASK, src/gpu_batch.rs:62-66)
  int nomask;
};

__device__ __forceinline__ float leaky(float v, float s) { return v < 0.0f ? v * s : v; }

// Prologue value of input element (row t of the input domain, channel c), given its item b >= 0.
// AdaIN arithmetic follows adain_apply_seg (kernels/kokoro.cu:317-334); Snake follows
// kernels/kokoro.cu:700-714 (x + (1/a) * sin(a x)^2).
__device__ __forceinline__ float prologue(const ConvArgs& a, float v, int b, int c) {
  if (a.in_mode == IN_ADAIN_LEAKY || a.in_mode == IN_ADAIN_SNAKE) {
    const int C = a.cin;
    v = (v - a.mean[b * C + c]) * a.rstd[b * C + c];
    const float* g = a.gb + (long)b * a.ldgb;
    float g1 = 1.0f + g[c];
    v = g1 * (v * a.nw[c] + a.nb[c]) + g[C + c];
    if (a.in_mode == IN_ADAIN_LEAKY) {
      v = leaky(v, a.slope);
    } else {
      float al = a.alpha[c];
      float inv = 1.0f / al;
      float sn = sinf(al * v);
      v = v + inv * (sn * sn);
    }
  } else if (a.in_mode == IN_LEAKY_MASK) {
    v = leaky(v, a.slope);
  }
  return v;
}

__device__ __forceinline__ float gelu_new(float a) {
  const float c = 0.797884560802865355f;  // (float)sqrt(2/pi), kernels/kokoro.cu:86
  return 0.5f * a * (1.0f + tanhf(c * (a + 0.044715f * a * a * a)));
}

}  // namespace kk
