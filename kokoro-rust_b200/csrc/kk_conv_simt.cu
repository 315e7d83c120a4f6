// fp32 SIMT implicit-GEMM 1-D convolution over the time-major ragged layout (FP32 precision
// mode). One kernel serves every convolution and linear layer of the forward:
//   y[t, co] = bias[co] + sum_k sum_ci W[k][ci][co] * P(x)[t*stride + k*dil - pad, ci]
// where P is the input prologue (gap masking, AdaIN + leaky ReLU, AdaIN + Snake, leaky ReLU)
// applied while the input window is staged, and the epilogue stores, accumulates (y +=),
// adds a shortcut and scales, or applies gelu_new. A linear layer is the K = 1 case; a
// ConvTranspose1d runs as its polyphase K-tap convolution with a [K][cin][s*cout] weight.
//
// Reference routes replaced: conv1d_wmma_bf16* (kernels/kokoro.cu:660-774), conv1d_strided
// (:549-617), conv_direct_tiled (:510-547), per-tap cuBLAS GEMMs and GLinear (src/gpu.rs:267-499),
// convT_gather + sgemm (src/gpu.rs:512-538), mask_gaps (:310), adain_apply_seg (:317).
#include "kk_common.cuh"
#include "kk_launch.h"

namespace kk {

constexpr int ST_TM = 64;   // time rows per block
constexpr int ST_TN = 64;   // output channels per block
constexpr int ST_CK = 16;   // input channels per stage

__global__ void __launch_bounds__(256) conv_simt_kernel(ConvArgs a) {
  extern __shared__ float smem[];
  const int tid = threadIdx.x;
  const int tx = tid & 15, ty = tid >> 4;
  const int t0 = blockIdx.x * ST_TM, co0 = blockIdx.y * ST_TN;
  const int win = (ST_TM - 1) * a.stride + (a.K - 1) * a.dil + 1;
  const int base = t0 * a.stride - a.pad;
  float* xs = smem;                      // [ST_CK][win]
  float* ws = smem + ST_CK * win;        // [K][ST_CK][ST_TN]
  float acc[4][4];
#pragma unroll
  for (int i = 0; i < 4; i++)
#pragma unroll
    for (int j = 0; j < 4; j++) acc[i][j] = 0.0f;

  for (int ci0 = 0; ci0 < a.cin; ci0 += ST_CK) {
    __syncthreads();
    for (int i = tid; i < ST_CK * win; i += 256) {
      int ci = i / win, j = i - ci * win;
      int c = ci0 + ci, r = base + j;
      float v = 0.0f;
      if (c < a.cin && r >= 0 && r < a.L_in) {
        if (a.in_mode == IN_NOMASK) {
          v = a.x[(long)(a.in_up2 ? (r >> 1) : r) * a.ldx + c];
        } else {
          int b = dom_item(a.din, r);
          if (b >= 0) v = prologue(a, a.x[(long)(a.in_up2 ? (r >> 1) : r) * a.ldx + c], b, c);
          else if (a.nomask) v = a.x[(long)(a.in_up2 ? (r >> 1) : r) * a.ldx + c];
        }
      }
      xs[i] = v;
    }
    const int nw = a.K * ST_CK * ST_TN;
    for (int i = tid; i < nw; i += 256) {
      int co = i & (ST_TN - 1), kc = i >> 6;
      int ci = kc % ST_CK, k = kc / ST_CK;
      int c = ci0 + ci, o = co0 + co;
      ws[i] = (c < a.cin && o < a.cout) ? a.w[((long)k * a.cin + c) * a.cout + o] : 0.0f;
    }
    __syncthreads();
    for (int k = 0; k < a.K; k++) {
      const float* xk = xs + k * a.dil + ty * 4 * a.stride;
      const float* wk = ws + k * ST_CK * ST_TN + tx * 4;
#pragma unroll 4
      for (int ci = 0; ci < ST_CK; ci++) {
        float xv[4];
#pragma unroll
        for (int i = 0; i < 4; i++) xv[i] = xk[ci * win + i * a.stride];
        float4 wv = *reinterpret_cast<const float4*>(wk + ci * ST_TN);
#pragma unroll
        for (int i = 0; i < 4; i++) {
          acc[i][0] = fmaf(xv[i], wv.x, acc[i][0]);
          acc[i][1] = fmaf(xv[i], wv.y, acc[i][1]);
          acc[i][2] = fmaf(xv[i], wv.z, acc[i][2]);
          acc[i][3] = fmaf(xv[i], wv.w, acc[i][3]);
        }
      }
    }
  }
#pragma unroll
  for (int i = 0; i < 4; i++) {
    int t = t0 + ty * 4 + i;
    if (t >= a.L_out) continue;
#pragma unroll
    for (int j = 0; j < 4; j++) {
      int co = co0 + tx * 4 + j;
      if (co >= a.cout) continue;
      float v = acc[i][j] + (a.bias ? a.bias[co] : 0.0f);
      long o = (long)t * a.ldy + co;
      switch (a.out_mode) {
        case OUT_ADD: v = a.y[o] + v; break;
        case OUT_PLUS: v = (v + a.sc[(long)t * a.ldsc + co]) * a.oscale; break;
        case OUT_GELU: v = gelu_new(v); break;
        default: break;
      }
      a.y[o] = v;
    }
  }
}

size_t conv_simt_smem(const ConvArgs& a) {
  int win = (ST_TM - 1) * a.stride + (a.K - 1) * a.dil + 1;
  return (size_t)(ST_CK * win + a.K * ST_CK * ST_TN) * sizeof(float);
}

cudaError_t launch_conv_simt(const ConvArgs& a, cudaStream_t st) {
  if (a.out_mode == OUT_GELU_PRE || a.out_mode == OUT_STORE_BF || a.x_b) return cudaErrorInvalidValue;  // tensor-core modes
  size_t smem = conv_simt_smem(a);
  static bool attr_set[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 64 && !attr_set[dev]) {
    cudaError_t e = cudaFuncSetAttribute(conv_simt_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);
    if (e != cudaSuccess) return e;
    attr_set[dev] = true;
  }
  if (smem > 200 * 1024) return cudaErrorInvalidValue;
  dim3 grid((a.L_out + ST_TM - 1) / ST_TM, (a.cout + ST_TN - 1) / ST_TN);
  conv_simt_kernel<<<grid, 256, smem, st>>>(a);
  return cudaGetLastError();
}

}  // namespace kk
