// Memory-bound and latency-bound kernels of the kokoro-b200 forward: embeddings, row
// LayerNorm / AdaLayerNorm, per-item attention (fp32), the persistent BiLSTM recurrence, AdaIN
// statistics, the AdaIN+pool upsampler, duration rounding, the F0/N curve convolutions, the
// harmonic source, STFT / iSTFT, and the small glue passes.
//
// Arithmetic that decides bit-level agreement with the reference is written out explicitly:
// the SineGen phase path uses the reference's FMA placement and f64 accumulation
// (kernels/kokoro.cu:188-254), durations use a sequential f32 sigmoid sum with
// round-half-to-even (src/model.rs:90-99), STFT / iSTFT run their DFTs in f64 (:470-508).
#include <cuda_bf16.h>
#include <math.h>
#include <string.h>
#include "kk_common.cuh"
#include "kk_launch.h"

namespace kk {

__constant__ double c_tw[440];  // [cos 11x20 | sin 11x20] of 2*pi*((k*n) % 20)/20 (src/gpu.rs:93-99)
__constant__ float c_win[20];   // periodic Hann(20) (src/gpu.rs:101)

static inline unsigned nblk(long n, int t) { return (unsigned)((n + t - 1) / t); }

// Sum of a double over a block of `blockDim.x` (multiple of 32, <= 1024) threads.
__device__ double block_sum_d(double v, double* sh) {
  for (int o = 16; o > 0; o >>= 1) v += __shfl_down_sync(0xffffffffu, v, o);
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31, nw = blockDim.x >> 5;
  __syncthreads();
  if (l == 0) sh[w] = v;
  __syncthreads();
  if (w == 0) {
    double r = l < nw ? sh[l] : 0.0;
    for (int o = 16; o > 0; o >>= 1) r += __shfl_down_sync(0xffffffffu, r, o);
    if (l == 0) sh[32] = r;
  }
  __syncthreads();
  return sh[32];
}

// ------------------------------------------------------------------------------ token side

__global__ void albert_embed_kernel(const int* ids, const int* row_item, const ItemTab* items, const float* word,
                                    const float* pos, const float* tt0, const float* g, const float* bb,
                                    float* out) {
  __shared__ double sh[33];
  const int r = blockIdx.x, j = threadIdx.x;  // 128 threads = EMB
  const int b = row_item[r];
  if (b < 0) {
    out[(long)r * 128 + j] = 0.0f;
    return;
  }
  const int i = r - items[b].tok_start;
  const int id = ids[r];
  const float v = __fadd_rn(__fadd_rn(word[id * 128 + j], tt0[j]), pos[i * 128 + j]);
  const float mean = (float)(block_sum_d((double)v, sh) / 128.0);
  const double c = (double)__fsub_rn(v, mean);
  const float var = (float)(block_sum_d(c * c, sh) / 128.0);
  const float inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(var, 1e-12f)));
  float o = __fmul_rn(__fsub_rn(v, mean), inv);
  o = __fadd_rn(__fmul_rn(o, g[j]), bb[j]);
  out[(long)r * 128 + j] = o;
}

cudaError_t launch_albert_embed(const int* ids, const int* row_item, const ItemTab* items, int rows,
                                const float* word, const float* pos, const float* tt0, const float* g,
                                const float* b, float* out, cudaStream_t st) {
  albert_embed_kernel<<<rows, 128, 0, st>>>(ids, row_item, items, word, pos, tt0, g, b, out);
  return cudaGetLastError();
}

__global__ void gather_rows_kernel(const float* src, int lds, const int* tab, int rows, int d, float* out, int ldo) {
  long i = blockIdx.x * (long)blockDim.x + threadIdx.x;
  if (i >= (long)rows * d) return;
  int r = (int)(i / d), j = (int)(i % d);
  int s = tab[r];
  out[(long)r * ldo + j] = s < 0 ? 0.0f : src[(long)s * lds + j];
}

// The same gather 16 bytes at a time (d, lds, ldo multiples of 4, aligned bases).
__global__ void gather_rows4_kernel(const float4* src, int lds4, const int* tab, int rows, int d4, float4* out,
                                    int ldo4) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= rows * d4) return;
  const int r = i / d4, j = i - r * d4;
  const int s = tab[r];
  out[(long)r * ldo4 + j] = s < 0 ? make_float4(0.0f, 0.0f, 0.0f, 0.0f) : __ldg(src + (long)s * lds4 + j);
}

cudaError_t launch_gather_rows(const float* src, int lds, const int* tab, int rows, int d, float* out, int ldo,
                               cudaStream_t st) {
  long n = (long)rows * d;
  if (n == 0) return cudaSuccess;
  if (d % 4 == 0 && lds % 4 == 0 && ldo % 4 == 0 && ((((uintptr_t)src) | ((uintptr_t)out)) & 15) == 0 &&
      n / 4 < (1L << 31)) {
    gather_rows4_kernel<<<nblk(n / 4, 256), 256, 0, st>>>((const float4*)src, lds / 4, tab, rows, d / 4, (float4*)out,
                                                          ldo / 4);
  } else {
    gather_rows_kernel<<<nblk(n, 256), 256, 0, st>>>(src, lds, tab, rows, d, out, ldo);
  }
  return cudaGetLastError();
}

// Projection of each row to a few channels (K = 1, cout <= 4; the F0 / N projections): one warp
// per row looks up the row's item once, its lanes read the row's channels (128 contiguous bytes
// per load) and a shuffle reduction sums the products; gap rows read nothing and give the bias.
__global__ void rowproj_kernel(const ConvArgs a) {
  const long r = (blockIdx.x * (long)blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (r >= a.L_out) return;
  const int b = a.in_mode == IN_NOMASK ? 0 : dom_item(a.din, (int)r);
  float acc[4] = {0.0f, 0.0f, 0.0f, 0.0f};
  if (b >= 0 || a.nomask) {
    const float* xr = a.x + r * a.ldx;
    for (int c = lane; c < a.cin; c += 32) {
      const float xv = __ldg(xr + c);
#pragma unroll
      for (int o = 0; o < 4; o++)
        if (o < a.cout) acc[o] = fmaf(xv, __ldg(a.w + (long)c * a.cout + o), acc[o]);
    }
  }
#pragma unroll
  for (int o = 0; o < 4; o++)
#pragma unroll
    for (int m = 16; m > 0; m >>= 1) acc[o] += __shfl_xor_sync(0xffffffffu, acc[o], m);
  if (lane == 0)
    for (int o = 0; o < a.cout; o++) a.y[r * a.ldy + o] = acc[o] + (a.bias ? a.bias[o] : 0.0f);
}

bool rowproj_supported(const ConvArgs& a) {
  return a.K == 1 && a.stride == 1 && a.cout >= 1 && a.cout <= 4 && !a.in_up2 && a.out_mode == OUT_STORE &&
         (a.in_mode == IN_MASK || a.in_mode == IN_NOMASK) && a.L_out == a.L_in;
}

cudaError_t launch_rowproj(const ConvArgs& a, cudaStream_t st) {
  if (!rowproj_supported(a)) return cudaErrorInvalidValue;
  if (a.L_out == 0) return cudaSuccess;
  rowproj_kernel<<<nblk((long)a.L_out * 32, 256), 256, 0, st>>>(a);
  return cudaGetLastError();
}

__global__ void embed_rows_kernel(const int* ids, const int* row_item, int rows, const float* table, int d, float* out) {
  long i = blockIdx.x * (long)blockDim.x + threadIdx.x;
  if (i >= (long)rows * d) return;
  int r = (int)(i / d), j = (int)(i % d);
  out[i] = row_item[r] < 0 ? 0.0f : table[(long)ids[r] * d + j];
}

// The same lookup 16 bytes at a time (d a multiple of 4, aligned table and output).
__global__ void embed_rows4_kernel(const int* ids, const int* row_item, int rows, const float4* table, int d4,
                                   float4* out) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= rows * d4) return;
  const int r = i / d4, j = i - r * d4;
  out[i] = row_item[r] < 0 ? make_float4(0.0f, 0.0f, 0.0f, 0.0f) : __ldg(table + (long)ids[r] * d4 + j);
}

cudaError_t launch_embed_rows(const int* ids, const int* row_item, int rows, const float* table, int d, float* out,
                              cudaStream_t st) {
  long n = (long)rows * d;
  if (n == 0) return cudaSuccess;
  if (d % 4 == 0 && ((((uintptr_t)table) | ((uintptr_t)out)) & 15) == 0 && n / 4 < (1L << 31))
    embed_rows4_kernel<<<nblk(n / 4, 256), 256, 0, st>>>(ids, row_item, rows, (const float4*)table, d / 4,
                                                         (float4*)out);
  else
    embed_rows_kernel<<<nblk(n, 256), 256, 0, st>>>(ids, row_item, rows, table, d, out);
  return cudaGetLastError();
}

__global__ void ln_rows_kernel(const float* x, int ldx, int d, const float* g, const float* bb, float eps, int mode,
                               float slope, const int* row_item, const float* gb, int ldgb, const float* style,
                               int sdim, float* y, int ldy) {
  __shared__ double sh[33];
  const int r = blockIdx.x;
  const float* row = x + (long)r * ldx;
  float* yr = y + (long)r * ldy;
  int item = 0;
  if (mode == 2) {
    item = row_item[r];
    if (item < 0) {
      for (int j = threadIdx.x; j < d + sdim; j += blockDim.x) yr[j] = 0.0f;
      return;
    }
  }
  double s = 0.0;
  for (int j = threadIdx.x; j < d; j += blockDim.x) s += (double)row[j];
  const float mean = (float)(block_sum_d(s, sh) / (double)d);
  double v = 0.0;
  for (int j = threadIdx.x; j < d; j += blockDim.x) {
    double c = (double)(row[j] - mean);
    v += c * c;
  }
  const float inv = 1.0f / sqrtf((float)(block_sum_d(v, sh) / (double)d) + eps);
  if (mode == 2) {
    const float* gg = gb + (long)item * ldgb;
    for (int j = threadIdx.x; j < d; j += blockDim.x) {
      float o = (row[j] - mean) * inv;
      yr[j] = (1.0f + gg[j]) * o + gg[d + j];
    }
    for (int j = threadIdx.x; j < sdim; j += blockDim.x) yr[d + j] = style[(long)item * sdim + j];
  } else {
    for (int j = threadIdx.x; j < d; j += blockDim.x) {
      float o = (row[j] - mean) * inv;
      if (g) o = o * g[j];
      if (bb) o = o + bb[j];
      if (mode == 1) o = leaky(o, slope);
      yr[j] = o;
    }
  }
}

// The same normalisation with one warp per row (d = 128 * NV, rows held in registers as float4):
// no block barriers, 8 rows per 256-thread block. Sums in double as above (the float mean and
// variance do not depend on the summation order).
__device__ __forceinline__ double warp_sum_d(double v) {
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

template <int NV>
__global__ void __launch_bounds__(256) ln_rows_warp_kernel(const float* x, int ldx, int rows, const float* g,
                                                           const float* bb, float eps, int mode, float slope,
                                                           const int* row_item, const float* gb, int ldgb,
                                                           const float* style, int sdim, float* y, int ldy,
                                                           uint8_t* ypre, long ypre_rows) {
  constexpr int d = 128 * NV;
  const int r = blockIdx.x * 8 + (threadIdx.x >> 5), lane = threadIdx.x & 31;
  if (r >= rows) return;
  const float4* row = reinterpret_cast<const float4*>(x + (long)r * ldx);
  float* yr = y + (long)r * ldy;
  int item = 0;
  if (mode == 2) {
    item = row_item[r];
    if (item < 0) {
      for (int j = lane; j < d + sdim; j += 32) yr[j] = 0.0f;
      return;
    }
  }
  float4 v[NV];
#pragma unroll
  for (int k = 0; k < NV; k++) v[k] = row[lane + 32 * k];
  double s = 0.0;
#pragma unroll
  for (int k = 0; k < NV; k++) s += ((double)v[k].x + (double)v[k].y) + ((double)v[k].z + (double)v[k].w);
  const float mean = (float)(warp_sum_d(s) / (double)d);
  double q = 0.0;
#pragma unroll
  for (int k = 0; k < NV; k++) {
    const double c0 = (double)(v[k].x - mean), c1 = (double)(v[k].y - mean);
    const double c2 = (double)(v[k].z - mean), c3 = (double)(v[k].w - mean);
    q += (c0 * c0 + c1 * c1) + (c2 * c2 + c3 * c3);
  }
  const float inv = 1.0f / sqrtf((float)(warp_sum_d(q) / (double)d) + eps);
  float4* yo = reinterpret_cast<float4*>(yr);
#pragma unroll
  for (int k = 0; k < NV; k++) {
    const int j = 4 * (lane + 32 * k);
    float o[4] = {(v[k].x - mean) * inv, (v[k].y - mean) * inv, (v[k].z - mean) * inv, (v[k].w - mean) * inv};
    if (mode == 2) {
      const float* gg = gb + (long)item * ldgb;
#pragma unroll
      for (int e = 0; e < 4; e++) o[e] = (1.0f + gg[j + e]) * o[e] + gg[d + j + e];
    } else {
#pragma unroll
      for (int e = 0; e < 4; e++) {
        if (g) o[e] = o[e] * g[j + e];
        if (bb) o[e] = o[e] + bb[j + e];
        if (mode == 1) o[e] = leaky(o[e], slope);
      }
    }
    yo[lane + 32 * k] = make_float4(o[0], o[1], o[2], o[3]);
    if (ypre) {  // channels j .. j + 3: half (j / 32) % 2 of chunk (j % 32) / 4 of block j / 64
      __nv_bfloat162 p0 = __floats2bfloat162_rn(o[0], o[1]), p1 = __floats2bfloat162_rn(o[2], o[3]);
      uint2 u;
      memcpy(&u.x, &p0, 4);
      memcpy(&u.y, &p1, 4);
      const int plane = (j >> 6) * 8 + ((j & 31) >> 2);
      *reinterpret_cast<uint2*>(ypre + ((size_t)plane * ypre_rows + PRE_PAD_FRONT + r) * 16 + ((j >> 5) & 1) * 8) = u;
    }
  }
  if (mode == 2)
    for (int j = lane; j < sdim; j += 32) yr[d + j] = style[(long)item * sdim + j];
}

cudaError_t launch_ln_rows(const float* x, int ldx, int rows, int d, const float* g, const float* b, float eps,
                           int mode, float slope, const int* row_item, const float* gb, int ldgb,
                           const float* style, int sdim, float* y, int ldy, cudaStream_t st, void* ypre,
                           long ypre_rows) {
  if (rows == 0) return cudaSuccess;
  const bool vec = ldx % 4 == 0 && ldy % 4 == 0 && (((uintptr_t)x | (uintptr_t)y) & 15) == 0;
  if (ypre && (!vec || mode == 2 || (d != 512 && d != 768) || (((uintptr_t)ypre) & 15) != 0))
    return cudaErrorInvalidValue;
  if (vec && (d == 512 || d == 768)) {
    const int grid = (rows + 7) / 8;
    if (d == 512)
      ln_rows_warp_kernel<4><<<grid, 256, 0, st>>>(x, ldx, rows, g, b, eps, mode, slope, row_item, gb, ldgb, style,
                                                   sdim, y, ldy, (uint8_t*)ypre, ypre_rows);
    else
      ln_rows_warp_kernel<6><<<grid, 256, 0, st>>>(x, ldx, rows, g, b, eps, mode, slope, row_item, gb, ldgb, style,
                                                   sdim, y, ldy, (uint8_t*)ypre, ypre_rows);
    return cudaGetLastError();
  }
  ln_rows_kernel<<<rows, 256, 0, st>>>(x, ldx, d, g, b, eps, mode, slope, row_item, gb, ldgb, style, sdim, y, ldy);
  return cudaGetLastError();
}

__global__ void cat_style_kernel(const int* row_item, int rows, int d, const float* style, int sdim, float* y, int ldy) {
  long i = blockIdx.x * (long)blockDim.x + threadIdx.x;
  const int w = d + sdim;
  if (i >= (long)rows * w) return;
  int r = (int)(i / w), j = (int)(i % w);
  int b = row_item[r];
  if (b < 0) y[(long)r * ldy + j] = 0.0f;
  else if (j >= d) y[(long)r * ldy + j] = style[(long)b * sdim + (j - d)];
}

cudaError_t launch_cat_style(const int* row_item, int rows, int d, const float* style, int sdim, float* y, int ldy,
                             cudaStream_t st) {
  long n = (long)rows * (d + sdim);
  cat_style_kernel<<<nblk(n, 256), 256, 0, st>>>(row_item, rows, d, style, sdim, y, ldy);
  return cudaGetLastError();
}

// Per-item 12-head attention, one thread per query row, keys/values staged 64 at a time,
// online softmax over blocks of 16 keys. qkv row: [q(768) | k(768) | v(768)], head h at h*64.
__global__ void __launch_bounds__(128) attention_f32_kernel(const float* qkv, int ld, const ItemTab* items,
                                                            float* ctx, int ldc) {
  __shared__ __align__(16) float Ks[64][64];
  __shared__ __align__(16) float Vs[64][64];
  const int b = blockIdx.x >> 2, qb = blockIdx.x & 3, h = blockIdx.y;
  const ItemTab it = items[b];
  const int T = it.tok_len;
  if (qb * 128 >= T) return;
  const int qi = qb * 128 + threadIdx.x;
  const bool valid = qi < T;
  float q[64], acc[64];
  float m = -INFINITY, l = 0.0f;
#pragma unroll
  for (int d = 0; d < 64; d++) {
    q[d] = valid ? qkv[(long)(it.tok_start + qi) * ld + h * 64 + d] : 0.0f;
    acc[d] = 0.0f;
  }
  for (int kb = 0; kb < T; kb += 64) {
    __syncthreads();
    for (int i = threadIdx.x; i < 64 * 64; i += 128) {
      int j = i >> 6, d = i & 63, row = kb + j;
      bool in = row < T;
      long base = (long)(it.tok_start + row) * ld + h * 64 + d;
      Ks[j][d] = in ? qkv[base + 768] : 0.0f;
      Vs[j][d] = in ? qkv[base + 1536] : 0.0f;
    }
    __syncthreads();
    if (!valid) continue;
    const int nk = min(64, T - kb);
    for (int j0 = 0; j0 < nk; j0 += 16) {
      float s[16];
      float mx = m;
#pragma unroll
      for (int jj = 0; jj < 16; jj++) {
        const int j = j0 + jj;
        float dot = 0.0f;
        if (j < nk) {
#pragma unroll
          for (int d = 0; d < 64; d += 4) {
            float4 kv = *reinterpret_cast<const float4*>(&Ks[j][d]);
            dot = fmaf(q[d], kv.x, dot);
            dot = fmaf(q[d + 1], kv.y, dot);
            dot = fmaf(q[d + 2], kv.z, dot);
            dot = fmaf(q[d + 3], kv.w, dot);
          }
          s[jj] = dot * 0.125f;
        } else {
          s[jj] = -INFINITY;
        }
        mx = fmaxf(mx, s[jj]);
      }
      if (mx > m) {
        const float corr = expf(m - mx);
        l *= corr;
#pragma unroll
        for (int d = 0; d < 64; d++) acc[d] *= corr;
        m = mx;
      }
#pragma unroll
      for (int jj = 0; jj < 16; jj++) {
        const float p = expf(s[jj] - m);
        l += p;
        if (j0 + jj < nk) {
#pragma unroll
          for (int d = 0; d < 64; d += 4) {
            float4 vv = *reinterpret_cast<const float4*>(&Vs[j0 + jj][d]);
            acc[d] = fmaf(p, vv.x, acc[d]);
            acc[d + 1] = fmaf(p, vv.y, acc[d + 1]);
            acc[d + 2] = fmaf(p, vv.z, acc[d + 2]);
            acc[d + 3] = fmaf(p, vv.w, acc[d + 3]);
          }
        }
      }
    }
  }
  if (valid) {
    const float inv = 1.0f / l;
    float* o = ctx + (long)(it.tok_start + qi) * ldc + h * 64;
#pragma unroll
    for (int d = 0; d < 64; d++) o[d] = acc[d] * inv;
  }
}

cudaError_t launch_attention_f32(const float* qkv, int ldqkv, const ItemTab* items, int B, int max_len, float* ctx,
                                 int ldc, cudaStream_t st) {
  (void)max_len;
  dim3 grid(B * 4, 12);
  attention_f32_kernel<<<grid, 128, 0, st>>>(qkv, ldqkv, items, ctx, ldc);
  return cudaGetLastError();
}

// ------------------------------------------------------------------------------ AdaIN statistics

// Block (item b, 128-channel group, row chunk): thread (float4 lane cl = 4 channels, row lane lr of
// 8) accumulates shifted f32 sums of its 4 channels over rows r0 + lr, r0 + lr + 8, ... with 4 rows
// in flight; the 8 row lanes are combined in shared memory and added to the item's f64 sums.
__global__ void __launch_bounds__(256) stats_partial_kernel(const float* x, int ldx, int C, const ItemTab* items,
                                                            int scale, int plus1, int chunk, double* part) {
  __shared__ float sh[8][32][8];
  const int b = blockIdx.x, cl = threadIdx.x & 31, lr = threadIdx.x >> 5;
  const int c0 = blockIdx.y * 128 + 4 * cl;
  const ItemTab it = items[b];
  const long start = (long)it.a * scale;
  const int len = it.n * scale + plus1;
  const int r0 = blockIdx.z * chunk, r1 = min(len, r0 + chunk);
  float s[4] = {0, 0, 0, 0}, s2[4] = {0, 0, 0, 0};
  const bool vec = (ldx % 4) == 0 && ((((uintptr_t)x) & 15) == 0) && c0 + 4 <= C;
  if (c0 < C && r0 < r1) {
    float sf[4];
#pragma unroll
    for (int e = 0; e < 4; e++) sf[e] = c0 + e < C ? x[start * ldx + c0 + e] : 0.0f;
    int r = r0 + lr;
    for (; r + 24 < r1; r += 32) {  // 4 rows in flight
      float v[4][4];
#pragma unroll
      for (int u = 0; u < 4; u++) {
        const float* p = x + (start + r + 8 * u) * ldx + c0;
        if (vec) {
          const float4 q = __ldg(reinterpret_cast<const float4*>(p));
          v[u][0] = q.x, v[u][1] = q.y, v[u][2] = q.z, v[u][3] = q.w;
        } else {
#pragma unroll
          for (int e = 0; e < 4; e++) v[u][e] = c0 + e < C ? __ldg(p + e) : 0.0f;
        }
      }
#pragma unroll
      for (int u = 0; u < 4; u++)
#pragma unroll
        for (int e = 0; e < 4; e++) {
          const float d = v[u][e] - sf[e];
          s[e] += d;
          s2[e] += d * d;
        }
    }
    for (; r < r1; r += 8) {
      const float* p = x + (start + r) * ldx + c0;
#pragma unroll
      for (int e = 0; e < 4; e++) {
        const float d = (c0 + e < C ? __ldg(p + e) : 0.0f) - sf[e];
        s[e] += d;
        s2[e] += d * d;
      }
    }
  }
#pragma unroll
  for (int e = 0; e < 4; e++) sh[lr][cl][e] = s[e], sh[lr][cl][4 + e] = s2[e];
  __syncthreads();
  if (threadIdx.x < 128) {
    const int c = blockIdx.y * 128 + threadIdx.x;  // one channel per thread
    const int l2 = threadIdx.x >> 2, e = threadIdx.x & 3;
    if (c < C && r0 < r1) {
      double S = 0.0, S2 = 0.0;
      for (int k = 0; k < 8; k++) {
        S += sh[k][l2][e];
        S2 += sh[k][l2][4 + e];
      }
      atomicAdd(part + ((long)b * C + c) * 2, S);
      atomicAdd(part + ((long)b * C + c) * 2 + 1, S2);
    }
  }
}

__global__ void stats_final_kernel(const float* x, int ldx, int C, const ItemTab* items, int B, int scale, int plus1,
                                   const double* part, float* mean, float* rstd) {
  int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= B * C) return;
  int b = i / C, c = i % C;
  const ItemTab it = items[b];
  const int len = it.n * scale + plus1;
  const float shift = x[(long)it.a * scale * ldx + c];
  double d = part[2L * i] / (double)len;
  double var = part[2L * i + 1] / (double)len - d * d;
  if (var < 0.0) var = 0.0;
  mean[i] = (float)((double)shift + d);
  rstd[i] = 1.0f / sqrtf((float)var + 1e-5f);
}

cudaError_t launch_stats(const float* x, int ldx, int C, const ItemTab* items, int B, int scale, int plus1,
                         int max_len, double* part, float* mean, float* rstd, cudaStream_t st) {
  cudaError_t e = cudaMemsetAsync(part, 0, sizeof(double) * 2L * B * C, st);
  if (e != cudaSuccess) return e;
  const int cg = (C + 127) / 128;
  const int chunk = 2048;  // rows per block: long frame-domain items are split over many blocks
  const int rs = max(1, (max_len + chunk - 1) / chunk);
  stats_partial_kernel<<<dim3(B, cg, rs), 256, 0, st>>>(x, ldx, C, items, scale, plus1, chunk, part);
  if ((e = cudaGetLastError()) != cudaSuccess) return e;
  stats_final_kernel<<<nblk((long)B * C, 256), 256, 0, st>>>(x, ldx, C, items, B, scale, plus1, part, mean, rstd);
  return cudaGetLastError();
}

__global__ void stats_from_sums_kernel(const double* part, int C, const ItemTab* items, int B, int scale, int plus1,
                                      float* mean, float* rstd) {
  int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= B * C) return;
  const ItemTab it = items[i / C];
  const double n = (double)(it.n * scale + plus1);
  const double m = part[2L * i] / n;
  double var = part[2L * i + 1] / n - m * m;
  if (var < 0.0) var = 0.0;
  mean[i] = (float)m;
  rstd[i] = 1.0f / sqrtf((float)var + 1e-5f);
}

cudaError_t launch_stats_from_sums(const double* part, int C, const ItemTab* items, int B, int scale, int plus1,
                                   float* mean, float* rstd, cudaStream_t st) {
  stats_from_sums_kernel<<<nblk((long)B * C, 256), 256, 0, st>>>(part, C, items, B, scale, plus1, mean, rstd);
  return cudaGetLastError();
}

__global__ void adain_coef_kernel(const float* mean, const float* rstd, const float* nw, const float* nb,
                                  const float* gb, int ldgb, int B, int C, float2* coef) {
  int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= B * C) return;
  int b = i / C, c = i % C;
  const float* g = gb + (long)b * ldgb;
  float g1 = 1.0f + g[c];
  float s = rstd[i] * nw[c];
  coef[i] = make_float2(g1 * s, g1 * (nb[c] - mean[i] * s) + g[C + c]);
}

cudaError_t launch_adain_coef(const float* mean, const float* rstd, const float* nw, const float* nb, const float* gb,
                              int ldgb, int B, int C, float2* coef, cudaStream_t st) {
  adain_coef_kernel<<<nblk((long)B * C, 256), 256, 0, st>>>(mean, rstd, nw, nb, gb, ldgb, B, C, coef);
  return cudaGetLastError();
}

// ------------------------------------------------------------------------------ AdaIN + pool

__device__ __forceinline__ float pool_in(const ConvArgs& p, const float* x, int L, int i, int c) {
  if (i < 0 || i >= L) return 0.0f;
  int b = dom_item(p.din, i);
  if (b < 0) return 0.0f;
  return prologue(p, x[(long)i * p.ldx + c], b, c);
}

__global__ void adain_pool_kernel(const float* x, int C, int L, ConvArgs p, const float* pw, const float* pb, float* y,
                                  int ldy) {
  long idx = blockIdx.x * (long)blockDim.x + threadIdx.x;
  if (idx >= 2L * L * C) return;
  int o = (int)(idx / C), c = (int)(idx % C);
  float acc = pb[c];
  if ((o & 1) == 0) {
    acc = fmaf(pw[c * 3 + 1], pool_in(p, x, L, o >> 1, c), acc);
  } else {
    acc = fmaf(pw[c * 3 + 2], pool_in(p, x, L, (o - 1) >> 1, c), acc);
    acc = fmaf(pw[c * 3 + 0], pool_in(p, x, L, (o + 1) >> 1, c), acc);
  }
  y[(long)o * ldy + c] = acc;
}

// The same AdaIN + leaky + depthwise transposed conv for the AdaIN-leaky prologue, organised by
// input row: thread = channel, block = 32 consecutive input rows. Each input value is transformed
// once (instead of once per output that reads it) and feeds output rows 2i (tap 1), 2i - 1 (tap 0)
// and 2i + 1 (tap 2); the item's AdaIN terms stay in registers while the item is unchanged. Rows
// go in chunks of 8: the items and input values of a chunk's 9 rows (8 + the next one) are all
// loaded before any is used, so each thread has 9 loads in flight instead of one (the pass is bound
// by memory latency otherwise). The arithmetic of every output is the one above, operation for
// operation.
constexpr int POOL_RB = 32;
constexpr int POOL_CH = 8;  // rows per chunk
__global__ void __launch_bounds__(256) adain_pool_rows_kernel(const float* __restrict__ x, int C, int L, ConvArgs p,
                                                              const float* __restrict__ pw,
                                                              const float* __restrict__ pb, float* __restrict__ y,
                                                              int ldy) {
  const int c = blockIdx.y * blockDim.x + threadIdx.x;
  if (c >= C) return;
  const int i0 = blockIdx.x * POOL_RB;
  const float w0 = pw[c * 3 + 0], w1 = pw[c * 3 + 1], w2 = pw[c * 3 + 2], bias = pb[c];
  const float nw = p.nw[c], nb = p.nb[c];
  int cached = -1;
  float mean = 0.0f, rstd = 0.0f, g1 = 0.0f, gc = 0.0f;
  for (int k0 = 0; k0 < POOL_RB && i0 + k0 < L; k0 += POOL_CH) {
    int bv[POOL_CH + 1];
    float xv[POOL_CH + 1];
#pragma unroll
    for (int u = 0; u <= POOL_CH; u++) {
      const int i = i0 + k0 + u;
      bv[u] = i < L ? dom_item(p.din, i) : -1;
    }
#pragma unroll
    for (int u = 0; u <= POOL_CH; u++) {
      const int i = i0 + k0 + u;
      xv[u] = bv[u] >= 0 ? x[(long)i * p.ldx + c] : 0.0f;
    }
    float uu[POOL_CH + 1];  // pool_in(p, x, L, i, c) of the chunk's rows
#pragma unroll
    for (int u = 0; u <= POOL_CH; u++) {
      const int b = bv[u];
      if (b < 0) {
        uu[u] = 0.0f;
        continue;
      }
      if (b != cached) {
        cached = b;
        mean = p.mean[b * C + c];
        rstd = p.rstd[b * C + c];
        const float* g = p.gb + (long)b * p.ldgb;
        g1 = 1.0f + g[c];
        gc = g[C + c];
      }
      float v = (xv[u] - mean) * rstd;
      v = g1 * (v * nw + nb) + gc;
      uu[u] = leaky(v, p.slope);
    }
#pragma unroll
    for (int u = 0; u < POOL_CH; u++) {
      const int i = i0 + k0 + u;
      if (i >= L) break;
      y[(long)(2 * i) * ldy + c] = fmaf(w1, uu[u], bias);
      float acc = fmaf(w2, uu[u], bias);
      acc = fmaf(w0, uu[u + 1], acc);
      y[(long)(2 * i + 1) * ldy + c] = acc;
    }
  }
}

cudaError_t launch_adain_pool(const float* x, int C, int L, const ConvArgs& pro, const float* pw, const float* pb,
                              float* y, int ldy, cudaStream_t st) {
  if (pro.in_mode == IN_ADAIN_LEAKY) {
    adain_pool_rows_kernel<<<dim3((unsigned)((L + POOL_RB - 1) / POOL_RB), (unsigned)((C + 255) / 256)), 256, 0, st>>>(
        x, C, L, pro, pw, pb, y, ldy);
    return cudaGetLastError();
  }
  long n = 2L * L * C;
  adain_pool_kernel<<<nblk(n, 256), 256, 0, st>>>(x, C, L, pro, pw, pb, y, ldy);
  return cudaGetLastError();
}

// ------------------------------------------------------------------------------ durations

__global__ void durations_kernel(const float* logits, int ldl, const int* row_item, const float* speed, int rows,
                                 int* dur, float* q) {
  int r = blockIdx.x * blockDim.x + threadIdx.x;
  if (r >= rows) return;
  int b = row_item[r];
  if (b < 0) {
    dur[r] = 0;
    q[r] = 0.0f;
    return;
  }
  const float* l = logits + (long)r * ldl;
  float s = 0.0f;
  for (int j = 0; j < 50; j++) s = __fadd_rn(s, __fdiv_rn(1.0f, __fadd_rn(1.0f, expf(-l[j]))));
  float v = __fdiv_rn(s, speed[b]);
  int d = (int)rintf(v);
  dur[r] = d < 1 ? 1 : d;
  q[r] = v;
}

cudaError_t launch_durations(const float* logits, int ldl, const int* row_item, const float* speed, int rows,
                             int* dur, float* q, cudaStream_t st) {
  durations_kernel<<<nblk(rows, 256), 256, 0, st>>>(logits, ldl, row_item, speed, rows, dur, q);
  return cudaGetLastError();
}

// ------------------------------------------------------------------------------ F0 / N curve convs

__device__ __forceinline__ float curve_at(const float* v, const Dom& d2, int i) {
  return dom_item(d2, i) >= 0 ? v[i] : 0.0f;
}

__global__ void curve_conv_kernel(const float* f0, const float* nc, Dom d2, int LN, CurveConv wf, CurveConv wn,
                                  float* dst0, int ld0, int col0, float* dst1, int ld1, int col1, float* dst2,
                                  int ld2, int col2) {
  int o = blockIdx.x * blockDim.x + threadIdx.x;
  if (o >= LN) return;
  float af = 0.0f, an = 0.0f;
  for (int k = 0; k < 3; k++) {
    int i = 2 * o + k - 1;
    af = fmaf(wf.w[k], curve_at(f0, d2, i), af);
    an = fmaf(wn.w[k], curve_at(nc, d2, i), an);
  }
  af = af + wf.b;
  an = an + wn.b;
  if (dst0) { dst0[(long)o * ld0 + col0] = af; dst0[(long)o * ld0 + col0 + 1] = an; }
  if (dst1) { dst1[(long)o * ld1 + col1] = af; dst1[(long)o * ld1 + col1 + 1] = an; }
  if (dst2) { dst2[(long)o * ld2 + col2] = af; dst2[(long)o * ld2 + col2 + 1] = an; }
}

cudaError_t launch_curve_conv(const float* f0, const float* nc, Dom d2, int LN, CurveConv wf, CurveConv wn,
                              float* dst0, int ld0, int col0, float* dst1, int ld1, int col1, float* dst2, int ld2,
                              int col2, cudaStream_t st) {
  curve_conv_kernel<<<nblk(LN, 256), 256, 0, st>>>(f0, nc, d2, LN, wf, wn, dst0, ld0, col0, dst1, ld1, col1, dst2,
                                                   ld2, col2);
  return cudaGetLastError();
}

// ------------------------------------------------------------------------------ harmonic source

__device__ __forceinline__ float torch_remainder1(float a) {
  float m = fmodf(a, 1.0f);
  if (m != 0.0f && m < 0.0f) m = m + 1.0f;
  return m;
}

// rad value of harmonic h at sample t of an item's F0 curve f0c [L] (upsampled nearest x300)
__device__ __forceinline__ float sine_rad(const float* f0c, int L, float near_scale, int t, int h) {
  int src = (int)floorf(__fmul_rn((float)t, near_scale));
  if (src > L - 1) src = L - 1;
  return torch_remainder1(__fdiv_rn(__fmul_rn(f0c[src], (float)(h + 1)), 24000.0f));
}

// phase_pre [h][2N domain]: linear downsample of rad by 300, f64 cumulative sum, * 2 pi * 300
// (sine_phase_pre, kernels/kokoro.cu:206-226). One thread per (item, harmonic).
__global__ void sine_phase_kernel(const float* f0, int L2, const ItemTab* items, int B, float* pp) {
  int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= B * 9) return;
  const int b = i / 9, h = i % 9;
  const ItemTab it = items[b];
  const int L = 2 * it.n, S = 300 * L, D = L;
  const float* f0c = f0 + 2L * it.a;
  float* out = pp + (long)h * L2 + 2L * it.a;
  const float near_scale = (float)(1.0 / 300.0);
  const float down_scale = (float)(1.0 / (1.0 / 300.0));
  double acc = 0.0;
  for (int d = 0; d < D; d++) {
    float real = fmaf(down_scale, __fadd_rn((float)d, 0.5f), -0.5f);
    if (real < 0.0f) real = 0.0f;
    int i0 = (int)floorf(real);
    if (i0 > S - 1) i0 = S - 1;
    float l1 = fminf(fmaxf(__fsub_rn(real, (float)i0), 0.0f), 1.0f);
    int i1 = i0 < S - 1 ? i0 + 1 : i0;
    float l0 = __fsub_rn(1.0f, l1);
    float v = fmaf(sine_rad(f0c, L, near_scale, i0, h), l0, __fmul_rn(sine_rad(f0c, L, near_scale, i1, h), l1));
    acc += (double)v;
    out[d] = __fmul_rn(__fmul_rn(__fmul_rn((float)acc, 2.0f), 3.14159274101257324f), 300.0f);
  }
}

cudaError_t launch_sine_phase(const float* f0, int L2, const ItemTab* items, int B, float* pp, cudaStream_t st) {
  sine_phase_kernel<<<nblk((long)B * 9, 64), 64, 0, st>>>(f0, L2, items, B, pp);
  return cudaGetLastError();
}

__device__ __forceinline__ unsigned long long splitmix_at(unsigned long long seed, unsigned long long ctr) {
  unsigned long long x = seed + (ctr + 1ULL) * 0x9E3779B97F4A7C15ULL;
  x = (x ^ (x >> 30)) * 0xBF58476D1CE4E5B9ULL;
  x = (x ^ (x >> 27)) * 0x94D049BB133111EBULL;
  return x ^ (x >> 31);
}

// har[t] = tanh(sum_h lw[h] * (sin(phase(t, h)) * 0.1 * uv + amp * noise[t*9 + h]) + lb)
// (sine_har_source + gen_noise, kernels/kokoro.cu:228-254, 282-302), noise generated in place
// from the item's counter stream or read from replayed draws (items whose noise_off is -1 use the
// counter stream, so one batch can mix both). One thread per sample of the 600N
// domain; gap samples -> 0. sin / tanh / log / sqrt / cos are evaluated in f64 and rounded once
// to f32 (correctly rounded results), so the source is reproducible on any IEEE CPU.
__global__ void har_source_kernel(const float* f0, const float* pp, int L2, const ItemTab* items,
                                  const int* col_item_n, int LN, const uint64_t* seeds, const float* noise,
                                  const long long* noise_off, const float* lw, float lb, float* har) {
  long c = blockIdx.x * (long)blockDim.x + threadIdx.x;
  if (c >= 600L * LN) return;
  const int b = col_item_n[c / 600];
  if (b < 0) {
    har[c] = 0.0f;
    return;
  }
  const ItemTab it = items[b];
  const int t = (int)(c - 600L * it.a);
  const int L = 2 * it.n, D = L;
  const float* f0c = f0 + 2L * it.a;
  const float near_scale = (float)(1.0 / 300.0);
  const float up_scale = (float)(1.0 / 300.0);
  int src = (int)floorf(__fmul_rn((float)t, near_scale));
  if (src > L - 1) src = L - 1;
  const float f0v = f0c[src];
  const float uv = f0v > 10.0f ? 1.0f : 0.0f;
  const float amp = __fadd_rn(__fmul_rn(uv, 0.003f), __fdiv_rn(__fmul_rn(__fsub_rn(1.0f, uv), 0.1f), 3.0f));
  float real = fmaf(up_scale, __fadd_rn((float)t, 0.5f), -0.5f);
  if (real < 0.0f) real = 0.0f;
  int i0 = (int)floorf(real);
  if (i0 > D - 1) i0 = D - 1;
  const float l1 = fminf(fmaxf(__fsub_rn(real, (float)i0), 0.0f), 1.0f);
  const int i1 = i0 < D - 1 ? i0 + 1 : i0;
  const float l0 = __fsub_rn(1.0f, l1);
  float nz[9];
  if (noise && noise_off[b] >= 0) {  // replayed draws (ItemNoise::Fixed); offset -1: the counter stream
    const float* nb = noise + noise_off[b] + (long)t * 9;
#pragma unroll
    for (int h = 0; h < 9; h++) nz[h] = nb[h];
  } else {
    const unsigned long long seed = seeds ? seeds[b] : 0ULL;
    const long q0 = (long)t * 9;
    for (long p = q0 >> 1; p <= (q0 + 8) >> 1; p++) {
      unsigned long long x = splitmix_at(seed, 1024ULL + (unsigned long long)p);
      float u1 = (float)((x >> 40) + 1ULL) * (1.0f / 16777216.0f);
      float u2 = (float)((x >> 16) & 0xFFFFFFULL) * (1.0f / 16777216.0f);
      float r = (float)sqrt(-2.0 * log((double)u1));
      float th = __fmul_rn(6.2831855f, u2);
      long e0 = 2 * p - q0, e1 = e0 + 1;
      double sd, cd;  // one argument reduction for both (the same values as cos() and sin())
      sincos((double)th, &sd, &cd);
      if (e0 >= 0 && e0 < 9) nz[e0] = __fmul_rn(r, (float)cd);
      if (e1 >= 0 && e1 < 9) nz[e1] = __fmul_rn(r, (float)sd);
    }
  }
  const float* ppb = pp + 2L * it.a;
  float acc = 0.0f;
#pragma unroll
  for (int h = 0; h < 9; h++) {
    const float* ph_row = ppb + (long)h * L2;
    float ph = fmaf(ph_row[i0], l0, __fmul_rn(ph_row[i1], l1));
    float sine = __fmul_rn((float)sin((double)ph), 0.1f);
    float v = __fadd_rn(__fmul_rn(sine, uv), __fmul_rn(amp, nz[h]));
    acc = __fadd_rn(acc, __fmul_rn(lw[h], v));
  }
  har[c] = (float)tanh((double)__fadd_rn(acc, lb));
}

cudaError_t launch_har_source(const float* f0, const float* pp, int L2, const ItemTab* items, const int* col_item_n,
                              int LN, const uint64_t* seeds, const float* noise, const long long* noise_off,
                              const float* lw, float lb, float* har, cudaStream_t st) {
  long n = 600L * LN;
  har_source_kernel<<<nblk(n, 256), 256, 0, st>>>(f0, pp, L2, items, col_item_n, LN, seeds, noise, noise_off, lw, lb,
                                                  har);
  return cudaGetLastError();
}

// ------------------------------------------------------------------------------ STFT / iSTFT

// One thread per frame row of the 120N+1 domain: reflect-padded centred window of the item's
// har, periodic Hann, f64 DFT -> magnitude and phase, 11 bins each (stft20_ld,
// kernels/kokoro.cu:470-490). The DFT accumulates sequentially without fused multiply-adds and
// magnitude / phase are evaluated in f64 and rounded once, so a CPU restatement reproduces the
// spectrum bit for bit: the phase channel is discontinuous at +-pi (atan2 branch cut) and the
// noise convolutions consume it linearly, so a one-ulp difference in a near-zero bin would
// otherwise move that bin by 2 pi. Gap rows -> 0.
__global__ void stft_kernel(const float* har, const ItemTab* items, Dom d120, float* spec, int lds) {
  int R = blockIdx.x * blockDim.x + threadIdx.x;
  if (R >= d120.L) return;
  float* out = spec + (long)R * lds;
  for (int k = 22; k < lds; k++) out[k] = 0.0f;  // row padding (read by the 6-frame-row view)
  int b = dom_item(d120, R);
  if (b < 0) {
    for (int k = 0; k < 22; k++) out[k] = 0.0f;
    return;
  }
  const ItemTab it = items[b];
  const int f = R - 120 * it.a;
  const int L = 600 * it.n;
  const float* x = har + 600L * it.a;
  double buf[20];
#pragma unroll
  for (int n = 0; n < 20; n++) {
    int p = f * 5 + n - 10;
    int src = p < 0 ? -p : (p >= L ? 2 * L - 2 - p : p);
    buf[n] = (double)(x[src] * c_win[n]);
  }
  for (int k = 0; k < 11; k++) {
    double re = 0.0, im = 0.0;
#pragma unroll
    for (int n = 0; n < 20; n++) {
      re = __dadd_rn(re, __dmul_rn(buf[n], c_tw[k * 20 + n]));
      im = __dsub_rn(im, __dmul_rn(buf[n], c_tw[220 + k * 20 + n]));
    }
    if (k == 0 || k == 10) im = 0.0;
    float rf = (float)re, imf = (float)im;
    out[k] = (float)hypot((double)rf, (double)imf);
    out[11 + k] = (float)atan2((double)imf, (double)rf);
  }
}

cudaError_t launch_stft(const float* har, const ItemTab* items, Dom d120, float* spec, int lds, cudaStream_t st) {
  stft_kernel<<<nblk(d120.L, 128), 128, 0, st>>>(har, items, d120, spec, lds);
  return cudaGetLastError();
}

// Fused iSTFT: a block owns 640 output samples; it first builds the windowed inverse-DFT frames
// it needs (exp magnitude, sin phase, 20-point real inverse DFT in f64, * Hann) in shared memory,
// then overlap-adds them and divides by the window envelope (istft_frames_ld + istft_ola,
// kernels/kokoro.cu:264-280, 492-508). Gap samples -> 0.
constexpr int IS_SAMPLES = 640;
constexpr int IS_FRAMES = IS_SAMPLES / 5 + 5;

__global__ void __launch_bounds__(128) istft_kernel(const float* post, int ldp, const ItemTab* items, Dom d120,
                                                    const int* col_item_n, int LN, float* audio) {
  __shared__ double fr[IS_FRAMES][20];
  const long s0 = (long)blockIdx.x * IS_SAMPLES;
  const long R_lo = s0 - 9 <= 0 ? 0 : (s0 - 9 + 4) / 5;
  for (int rr = threadIdx.x; rr < IS_FRAMES; rr += blockDim.x) {
    const long R = R_lo + rr;
    if (R >= d120.L || dom_item(d120, (int)R) < 0) continue;
    const float* pv = post + R * ldp;
    double re[11], im[11];
#pragma unroll
    for (int k = 0; k < 11; k++) {
      float m = expf(pv[k]);
      float p = sinf(pv[11 + k]);
      re[k] = (double)(m * cosf(p));
      im[k] = (double)(m * sinf(p));
    }
#pragma unroll
    for (int n = 0; n < 20; n++) {
      double v = re[0] + re[10] * ((n % 2 == 0) ? 1.0 : -1.0);
#pragma unroll
      for (int k = 1; k < 10; k++) v += 2.0 * (re[k] * c_tw[k * 20 + n] - im[k] * c_tw[220 + k * 20 + n]);
      v = v / 20.0;
      fr[rr][n] = v * (double)c_win[n];
    }
  }
  __syncthreads();
  for (int e = threadIdx.x; e < IS_SAMPLES; e += blockDim.x) {
    const long s = s0 + e;
    if (s >= 600L * LN) break;
    const int b = col_item_n[s / 600];
    if (b < 0) {
      audio[s] = 0.0f;
      continue;
    }
    const ItemTab it = items[b];
    const int F = 120 * it.n + 1;
    const int j = (int)(s - 600L * it.a) + 10;
    const int f_lo = j - 19 > 0 ? (j - 19 + 4) / 5 : 0;
    const int f_hi = min(j / 5, F - 1);
    double acc = 0.0, env = 0.0;
    for (int f = f_lo; f <= f_hi; f++) {
      const int n = j - 5 * f;
      const long R = 120L * it.a + f;
      acc += fr[R - R_lo][n];
      const double w = (double)c_win[n];
      env += w * w;
    }
    audio[s] = (float)(acc / env);
  }
}

cudaError_t launch_istft(const float* post, int ldp, const ItemTab* items, Dom d120, const int* col_item_n, int LN,
                         float* audio, cudaStream_t st) {
  long n = 600L * LN;
  istft_kernel<<<nblk(n, IS_SAMPLES), 128, 0, st>>>(post, ldp, items, d120, col_item_n, LN, audio);
  return cudaGetLastError();
}

// ------------------------------------------------------------------------------ glue

__global__ void sum3_kernel(const float4* r0, const float4* r1, const float4* r2, float4* y, long n4) {
  long i = blockIdx.x * (long)blockDim.x + threadIdx.x;
  if (i >= n4) return;
  const float4 a = __ldg(r0 + i), b = __ldg(r1 + i), c = __ldg(r2 + i);
  y[i] = make_float4(((a.x + b.x) + c.x) / 3.0f, ((a.y + b.y) + c.y) / 3.0f, ((a.z + b.z) + c.z) / 3.0f,
                     ((a.w + b.w) + c.w) / 3.0f);
}

cudaError_t launch_sum3(const float* r0, const float* r1, const float* r2, float* y, long n, cudaStream_t st) {
  if (n % 4 != 0) return cudaErrorInvalidValue;  // channel counts of the generator are multiples of 4
  sum3_kernel<<<nblk(n / 4, 256), 256, 0, st>>>((const float4*)r0, (const float4*)r1, (const float4*)r2,
                                                 (float4*)y, n / 4);
  return cudaGetLastError();
}

// Stage-1 ReflectionPad1d((1, 0)) per item (reflect_pad_left1_seg, kernels/kokoro.cu:452-467)
// fused with the noise-branch add: x[o] = pad(y)[o] + xs[o]; y holds 120 N rows, x 120 N + 1.
// Block of 256 threads = 8 rows x 32 float4 lanes (C = 128 channels per row; wider C loops).
__global__ void reflect_add_kernel(const float* y, const float* xs, int C, const ItemTab* items, Dom d120, float* x) {
  const int o = blockIdx.x * 8 + (threadIdx.x >> 5);
  if (o >= d120.L) return;
  const int b = dom_item(d120, o);
  long src = -1;
  if (b >= 0) {
    const int s = 120 * items[b].a;
    src = (o == s) ? (long)(s + 1) : (long)(o - 1);
  }
  for (int c = 4 * (threadIdx.x & 31); c < C; c += 128) {
    float4 v = src >= 0 ? __ldg(reinterpret_cast<const float4*>(y + src * C + c)) : make_float4(0, 0, 0, 0);
    const float4 a = __ldg(reinterpret_cast<const float4*>(xs + (long)o * C + c));
    v.x += a.x, v.y += a.y, v.z += a.z, v.w += a.w;
    *reinterpret_cast<float4*>(x + (long)o * C + c) = v;
  }
}

cudaError_t launch_reflect_add(const float* y, const float* xs, int C, const ItemTab* items, Dom d120, float* x,
                               cudaStream_t st) {
  if (C % 4 != 0) return cudaErrorInvalidValue;
  reflect_add_kernel<<<(d120.L + 7) / 8, 256, 0, st>>>(y, xs, C, items, d120, x);
  return cudaGetLastError();
}

// The same for C = 128 with the AdaIN sums of the result (BF16 mode: plain f32 partial sums, as the
// tensor-core epilogue forms them, added into f64 part[(item * 128 + c) * 2 + {0, 1}]). Block =
// 8 warps over RS_ROWS consecutive rows (warp w: rows w, w + 8, ...), lane = 4 channels; a lane
// adds its partials when the row's item changes and at the end (items span thousands of rows).
constexpr int RS_ROWS = 2048;
__global__ void reflect_add_stats_kernel(const float* y, const float* xs, const ItemTab* items, Dom d120, float* x,
                                         double* part) {
  const int warp = threadIdx.x >> 5, c = 4 * (threadIdx.x & 31);
  const int r0 = blockIdx.x * RS_ROWS, r1 = min(d120.L, r0 + RS_ROWS);
  int cb = -1;
  float s[4] = {0.0f, 0.0f, 0.0f, 0.0f}, q[4] = {0.0f, 0.0f, 0.0f, 0.0f};
  auto flush = [&]() {
    if (cb >= 0)
#pragma unroll
      for (int e = 0; e < 4; e++) {
        atomicAdd(part + ((long)cb * 128 + c + e) * 2, (double)s[e]);
        atomicAdd(part + ((long)cb * 128 + c + e) * 2 + 1, (double)q[e]);
        s[e] = q[e] = 0.0f;
      }
  };
  for (int o = r0 + warp; o < r1; o += 8) {
    const int b = dom_item(d120, o);
    long src = -1;
    if (b >= 0) {
      const int st = 120 * items[b].a;
      src = (o == st) ? (long)(st + 1) : (long)(o - 1);
    }
    float4 v = src >= 0 ? __ldg(reinterpret_cast<const float4*>(y + src * 128 + c)) : make_float4(0, 0, 0, 0);
    const float4 a = __ldg(reinterpret_cast<const float4*>(xs + (long)o * 128 + c));
    v.x += a.x, v.y += a.y, v.z += a.z, v.w += a.w;
    *reinterpret_cast<float4*>(x + (long)o * 128 + c) = v;
    if (b != cb) {
      flush();
      cb = b;
    }
    if (b >= 0) {
      const float e4[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
      for (int e = 0; e < 4; e++) {
        s[e] += e4[e];
        q[e] = fmaf(e4[e], e4[e], q[e]);
      }
    }
  }
  flush();
}

cudaError_t launch_reflect_add_stats(const float* y, const float* xs, const ItemTab* items, Dom d120, float* x,
                                     double* part, cudaStream_t st) {
  if (d120.L == 0) return cudaSuccess;
  reflect_add_stats_kernel<<<(d120.L + RS_ROWS - 1) / RS_ROWS, 256, 0, st>>>(y, xs, items, d120, x, part);
  return cudaGetLastError();
}

// PCM_16 of every sample of the batch (src/wav.rs:76-84: s * 32767 rounded half to even, values
// outside [-32768, 32767] (and NaN, stored as 0) clamped and counted per item).
__global__ void pcm16_kernel(const float* audio, long n, const int* col_item_n, int16_t* out,
                             unsigned long long* clipped) {
  const long i = blockIdx.x * (long)blockDim.x + threadIdx.x;
  if (i >= n) return;
  const float v = rintf(audio[i] * 32767.0f);
  int16_t q;
  if (!(v >= -32768.0f && v <= 32767.0f)) {
    q = v != v ? 0 : (v < 0.0f ? -32768 : 32767);
    const int b = col_item_n[i / 600];
    if (b >= 0) atomicAdd(clipped + b, 1ull);
  } else {
    q = (int16_t)v;
  }
  out[i] = q;
}

cudaError_t launch_pcm16(const float* audio, long n, const int* col_item_n, int16_t* out, unsigned long long* clipped,
                         cudaStream_t st) {
  if (n == 0) return cudaSuccess;
  pcm16_kernel<<<nblk(n, 256), 256, 0, st>>>(audio, n, col_item_n, out, clipped);
  return cudaGetLastError();
}

__global__ void copy_cols_kernel(const float* src, int lds, int c0s, float* dst, int ldd, int c0d, int rows, int ncol) {
  long i = blockIdx.x * (long)blockDim.x + threadIdx.x;
  if (i >= (long)rows * ncol) return;
  int r = (int)(i / ncol), j = (int)(i % ncol);
  dst[(long)r * ldd + c0d + j] = src[(long)r * lds + c0s + j];
}

cudaError_t launch_copy_cols(const float* src, int lds, int c0s, float* dst, int ldd, int c0d, int rows, int ncol,
                             cudaStream_t st) {
  long n = (long)rows * ncol;
  if (n == 0) return cudaSuccess;
  copy_cols_kernel<<<nblk(n, 256), 256, 0, st>>>(src, lds, c0s, dst, ldd, c0d, rows, ncol);
  return cudaGetLastError();
}

cudaError_t upload_stft_constants(cudaStream_t st) {
  double tw[440];
  for (int k = 0; k < 11; k++)
    for (int n = 0; n < 20; n++) {
      double a = 2.0 * M_PI * (double)((k * n) % 20) / 20.0;
      tw[k * 20 + n] = cos(a);
      tw[220 + k * 20 + n] = sin(a);
    }
  float win[20];
  for (int n = 0; n < 20; n++) win[n] = (float)(0.5 - 0.5 * cos(2.0 * M_PI * (double)n / 20.0));
  cudaError_t e = cudaMemcpyToSymbolAsync(c_tw, tw, sizeof(tw), 0, cudaMemcpyHostToDevice, st);
  if (e != cudaSuccess) return e;
  e = cudaMemcpyToSymbolAsync(c_win, win, sizeof(win), 0, cudaMemcpyHostToDevice, st);
  if (e != cudaSuccess) return e;
  return cudaStreamSynchronize(st);
}

}  // namespace kk
