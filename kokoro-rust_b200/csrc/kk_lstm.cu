// Bidirectional LSTM recurrence on thread-block clusters (both precision modes; fp32 throughout).
//
// Semantics (kernels/kokoro.cu:400-450): per item and direction, h_0 = c_0 = 0 and per step
//   gates = gx_t + (W_hh h_{t-1} + b_hh), order i, f, g, o;  c = f c + i g;  h = o tanh(c),
// where gx_t = W_ih x_t + b_ih comes from one GEMM over all rows before the recurrence.
//
// Work split. Items (sorted longest-first) form groups of up to 32; one cluster of 8 CTAs runs one
// (group, direction). CTA `rank` owns hidden units [32 rank, 32 rank + 32): thread (unit ul, k-slice
// ks) keeps W_hh[4 gates][unit][32 ks .. 32 ks + 31] in registers for the whole sequence (128
// floats), so the only shared-memory traffic of the dot products is the broadcast hidden state.
// Each step, for every active item: 8-lane partial dot products with packed f32x2 FMAs (each lane
// rounds exactly like fmaf), an 8-lane butterfly reduction, and the cell update by one lane per
// (unit, item). The CTA's new 32-unit slice of every item's hidden state is then pushed into all 8
// CTAs' shared memory with distributed-shared-memory stores, and one hardware cluster barrier
// closes the step: no global-memory barrier, no polling, no re-staging of h from L2.
// Every CTA of a cluster executes the same number of steps and barriers (the active-item count is
// the same for the whole group), so the cluster barrier cannot wait on an absent CTA.
#include <cuda_runtime.h>
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>

#include "kk_launch.h"

namespace kk {

namespace {

constexpr int LC_CL = 8;                // CTAs per cluster: 8 slices of 32 hidden units
constexpr int LC_H = 256;               // hidden units per direction
constexpr int LC_SL = 36;               // floats per 32-unit slice of a staged hidden row (16-B aligned)
constexpr int LC_HROW = LC_CL * LC_SL;  // staged hidden row (288 floats)
constexpr int LC_TLD = 36;              // row stride of the exchange tile
constexpr int LC_IPG = 32;              // items per group
constexpr int LC_NB = LC_IPG / 8;       // batches of 8 items

__device__ __forceinline__ uint32_t cl_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
__device__ __forceinline__ void cluster_sync() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
__device__ __forceinline__ void st_cluster_v4(uint32_t local_addr, uint32_t rank, float4 v) {
  uint32_t ra;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(ra) : "r"(local_addr), "r"(rank));
  asm volatile("st.shared::cluster.v4.f32 [%0], {%1, %2, %3, %4};" ::"r"(ra), "f"(v.x), "f"(v.y), "f"(v.z),
               "f"(v.w)
               : "memory");
}
__device__ __forceinline__ float sigm(float x) { return 1.0f / (1.0f + expf(-x)); }

__global__ void __cluster_dims__(LC_CL, 1, 1) __launch_bounds__(256, 1) lstm_cluster_kernel(const LstmArgs a) {
  extern __shared__ __align__(16) float sm[];
  float* Hs = sm;                                    // [2][LC_IPG][LC_HROW] staged hidden states
  float* Tile = Hs + 2 * LC_IPG * LC_HROW;           // [LC_IPG][LC_TLD] this CTA's new slice
  float* Gp = Tile + LC_IPG * LC_TLD;                // [8 warps][4 units][8 items][4 gates]
  const int rank = (int)cl_rank();
  const int cl = blockIdx.x / LC_CL;
  const int dir = cl & 1, g = cl >> 1;
  const int tid = threadIdx.x, warp = tid >> 5;
  const int ul = tid >> 3, ks = tid & 7;
  const int u = rank * 32 + ul;

  // W_hh rows of unit u, gates (0, 1) and (2, 3) paired for f32x2 FMAs, k-slice ks
  float2 w01[32], w23[32];
  {
    const float* W = a.whh + (size_t)dir * 4 * LC_H * LC_H;
#pragma unroll
    for (int kk = 0; kk < 32; kk++) {
      const int k = ks * 32 + kk;
      w01[kk] = make_float2(W[(size_t)(0 * LC_H + u) * LC_H + k], W[(size_t)(1 * LC_H + u) * LC_H + k]);
      w23[kk] = make_float2(W[(size_t)(2 * LC_H + u) * LC_H + k], W[(size_t)(3 * LC_H + u) * LC_H + k]);
    }
  }
  float bh[4];
#pragma unroll
  for (int q = 0; q < 4; q++) bh[q] = a.bhh[dir * 4 * LC_H + q * LC_H + u];
  // items of this thread's cell updates (8 b + ks) and of its pushes (tid / 8)
  const int* gs = a.gstart + g * LC_IPG;
  const int* gl = a.glen + g * LC_IPG;
  int st_[LC_NB], ln_[LC_NB];
#pragma unroll
  for (int b = 0; b < LC_NB; b++) st_[b] = gs[8 * b + ks], ln_[b] = gl[8 * b + ks];
  const int pi = tid >> 3, pc = tid & 7;
  const int pst = gs[pi], pln = gl[pi];
  float c[LC_NB];
#pragma unroll
  for (int b = 0; b < LC_NB; b++) c[b] = 0.0f;
  for (int i = tid; i < LC_IPG * LC_HROW; i += 256) Hs[i] = 0.0f;  // h_0 = 0
  const int* act = a.gact + (long)g * a.Tmax;
  cluster_sync();  // every CTA of the cluster is running and initialised before remote stores

  for (int s = 0; s < a.Tmax; s++) {
    const int na = act[s];
    if (na == 0) break;  // same for the whole group, so for every CTA of the cluster
    const float* Hc = Hs + (s & 1) * LC_IPG * LC_HROW;
    float* Hn = Hs + ((s + 1) & 1) * LC_IPG * LC_HROW;
    // gate inputs of this thread's cell updates, loaded ahead of the dot products
    float gxv[LC_NB][4];
#pragma unroll
    for (int b = 0; b < LC_NB; b++) {
      const int i = 8 * b + ks;
#pragma unroll
      for (int q = 0; q < 4; q++) gxv[b][q] = 0.0f;
      if (i < na) {
        const int t = dir == 0 ? s : ln_[b] - 1 - s;
        const float* gp = a.gx + (long)(st_[b] + t) * a.ldgx + dir * 4 * LC_H + u;
#pragma unroll
        for (int q = 0; q < 4; q++) gxv[b][q] = __ldg(gp + q * LC_H);
      }
    }
    float* gpw = Gp + warp * 128 + (ul & 3) * 32;
#pragma unroll
    for (int b = 0; b < LC_NB; b++) {
      if (8 * b >= na) break;
      // items in pairs: four independent f32x2 FMA chains, then one 3-level reduce-scatter of the
      // pair's 8 partial sums (index item * 4 + gate) over the 8 k-slice lanes, after which lane ks
      // holds the full dot product of value index ks
#pragma unroll 2
      for (int j = 0; j < 8; j += 2) {
        const int i = 8 * b + j;
        if (i >= na) break;
        const float* ha = Hc + i * LC_HROW + ks * LC_SL;
        const float* hb = ha + LC_HROW;  // item i + 1 (a stale row when i + 1 >= na: never used)
        float2 a01 = make_float2(0.0f, 0.0f), a23 = a01, b01 = a01, b23 = a01;
#pragma unroll
        for (int k4 = 0; k4 < 8; k4++) {
          const float4 x = *reinterpret_cast<const float4*>(ha + 4 * k4);
          const float4 y = *reinterpret_cast<const float4*>(hb + 4 * k4);
          a01 = __ffma2_rn(w01[4 * k4 + 0], make_float2(x.x, x.x), a01);
          a23 = __ffma2_rn(w23[4 * k4 + 0], make_float2(x.x, x.x), a23);
          b01 = __ffma2_rn(w01[4 * k4 + 0], make_float2(y.x, y.x), b01);
          b23 = __ffma2_rn(w23[4 * k4 + 0], make_float2(y.x, y.x), b23);
          a01 = __ffma2_rn(w01[4 * k4 + 1], make_float2(x.y, x.y), a01);
          a23 = __ffma2_rn(w23[4 * k4 + 1], make_float2(x.y, x.y), a23);
          b01 = __ffma2_rn(w01[4 * k4 + 1], make_float2(y.y, y.y), b01);
          b23 = __ffma2_rn(w23[4 * k4 + 1], make_float2(y.y, y.y), b23);
          a01 = __ffma2_rn(w01[4 * k4 + 2], make_float2(x.z, x.z), a01);
          a23 = __ffma2_rn(w23[4 * k4 + 2], make_float2(x.z, x.z), a23);
          b01 = __ffma2_rn(w01[4 * k4 + 2], make_float2(y.z, y.z), b01);
          b23 = __ffma2_rn(w23[4 * k4 + 2], make_float2(y.z, y.z), b23);
          a01 = __ffma2_rn(w01[4 * k4 + 3], make_float2(x.w, x.w), a01);
          a23 = __ffma2_rn(w23[4 * k4 + 3], make_float2(x.w, x.w), a23);
          b01 = __ffma2_rn(w01[4 * k4 + 3], make_float2(y.w, y.w), b01);
          b23 = __ffma2_rn(w23[4 * k4 + 3], make_float2(y.w, y.w), b23);
        }
        // value index v = item * 4 + gate: [a.x a.y a.z a.w | b.x b.y b.z b.w]
        const bool h4 = ks & 4, h2 = ks & 2, h1 = ks & 1;
        // level 1 (xor 4): keep the item of bit 2, send the other
        float k0 = h4 ? b01.x : a01.x, k1 = h4 ? b01.y : a01.y, k2 = h4 ? b23.x : a23.x, k3 = h4 ? b23.y : a23.y;
        const float s0 = h4 ? a01.x : b01.x, s1 = h4 ? a01.y : b01.y, s2 = h4 ? a23.x : b23.x,
                    s3 = h4 ? a23.y : b23.y;
        k0 += __shfl_xor_sync(0xffffffffu, s0, 4);
        k1 += __shfl_xor_sync(0xffffffffu, s1, 4);
        k2 += __shfl_xor_sync(0xffffffffu, s2, 4);
        k3 += __shfl_xor_sync(0xffffffffu, s3, 4);
        // level 2 (xor 2): keep the gate pair of bit 1
        float m0 = h2 ? k2 : k0, m1 = h2 ? k3 : k1;
        const float t0 = h2 ? k0 : k2, t1 = h2 ? k1 : k3;
        m0 += __shfl_xor_sync(0xffffffffu, t0, 2);
        m1 += __shfl_xor_sync(0xffffffffu, t1, 2);
        // level 3 (xor 1): keep the gate of bit 0
        float r = h1 ? m1 : m0;
        const float t = h1 ? m0 : m1;
        r += __shfl_xor_sync(0xffffffffu, t, 1);
        gpw[(j + (ks >> 2)) * 4 + (ks & 3)] = r;
      }
      __syncwarp();
      // cell update of (unit u, item 8 b + ks)
      const int i = 8 * b + ks;
      const float4 gp = *reinterpret_cast<const float4*>(gpw + ks * 4);
      if (i < na) {
        const float ig = sigm(gxv[b][0] + (gp.x + bh[0]));
        const float fg = sigm(gxv[b][1] + (gp.y + bh[1]));
        const float cg = tanhf(gxv[b][2] + (gp.z + bh[2]));
        const float og = sigm(gxv[b][3] + (gp.w + bh[3]));
        c[b] = fg * c[b] + ig * cg;
        Tile[i * LC_TLD + ul] = og * tanhf(c[b]);
      }
      __syncwarp();  // Gp is rewritten by the next batch
    }
    __syncthreads();  // Tile holds this CTA's 32-unit slice of every active item's new h
    if (pi < na) {
      const float4 v = *reinterpret_cast<const float4*>(Tile + pi * LC_TLD + 4 * pc);
      const uint32_t la = (uint32_t)__cvta_generic_to_shared(Hn + pi * LC_HROW + rank * LC_SL + 4 * pc);
#pragma unroll
      for (int r = 0; r < LC_CL; r++) st_cluster_v4(la, (uint32_t)r, v);
      const int t = dir == 0 ? s : pln - 1 - s;
      *reinterpret_cast<float4*>(a.out + (long)(pst + t) * a.ldo + dir * LC_H + rank * 32 + 4 * pc) = v;
    }
    cluster_sync();  // step s + 1 reads Hn: every slice has arrived in every CTA
  }
}

}  // namespace

cudaError_t launch_lstm(const LstmArgs& a, cudaStream_t st) {
  if (a.Tmax == 0 || a.G == 0) return cudaSuccess;
  if (a.IPG != LC_IPG) return cudaErrorInvalidValue;
  const size_t smem = sizeof(float) * (2 * LC_IPG * LC_HROW + LC_IPG * LC_TLD + 8 * 128);
  static bool attr[64] = {false};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 64 && !attr[dev]) {
    cudaError_t e = cudaFuncSetAttribute(lstm_cluster_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
    attr[dev] = true;
  }
  if (getenv("KK_LSTM_INFO")) {  // diagnostics: how many clusters of this kernel fit the device at once
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(a.G * 2 * LC_CL);
    cfg.blockDim = dim3(256);
    cfg.dynamicSmemBytes = smem;
    int n = -1;
    cudaOccupancyMaxActiveClusters(&n, (const void*)lstm_cluster_kernel, &cfg);
    fprintf(stderr, "lstm: %d clusters launched, %d can be resident\n", a.G * 2, n);
  }
  lstm_cluster_kernel<<<dim3(a.G * 2 * LC_CL), dim3(256), smem, st>>>(a);
  return cudaGetLastError();
}

}  // namespace kk
