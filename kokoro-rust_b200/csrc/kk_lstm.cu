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

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <string.h>

#include "kk_launch.h"
#include "kk_tc_ptx.cuh"

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

// ------------------------------------------------------------------------------ tcgen05 variant
//
// BF16 precision mode. Same clusters, groups and cell arithmetic (the cell's sigmoid / tanh from the
// hardware exponential, within a few ulp of the fp32 functions); the
// recurrent product of a step, G[128 gate rows][32 items] = W_hh[rows of this CTA's 32 units][256] x
// H[256][32 items], runs on the tensor cores with fp32-level accuracy by the split-operand method
// published for tensor cores as "3xTF32" (CUTLASS), here with fp16 halves: each operand is split
// into a big and a scaled small fp16 part, x = hi + lo / 2^11 with hi = fp16(x) and
// lo = fp16((x - hi) * 2^11), so hi + lo carries 22 significant bits; the products of fp16 values are
// exact in the fp32 accumulator, and G = Wh Hh + (Wh Hl + Wl Hh) / 2^11, dropping Wl Hl / 2^22
// (2^-22 relative, next to fp32's 2^-24 rounding). The scaled small parts keep every piece in fp16's
// normal range (|h| < 1; the engine routes weights with |W| above 2^15 to the fp32 kernel). The H
// image of a step holds Hh in its rows 0..31 and Hl in rows 32..63, so each K step is two MMAs:
// Wh x [Hh | Hl] (N 64, columns 0..63) and Wl x Hh (N 32, accumulated into columns 32..63);
// G = columns 0..31 + columns 32..63 / 2^11. A rows are ordered unit * 4 + gate, so
// the four gates of a unit sit in four neighbouring TMEM lanes; a 4-lane transpose through shared
// memory hands each thread one unit's four gates for 4 items. Each thread writes its new h, split
// into fp16 big / scaled small parts, straight into this CTA's 4 KB slice of its own next H image
// (and to the output); one bulk copy per other CTA
// then sends the slice, completing bytes of the receiver's own mbarrier: each CTA waits (bounded)
// for the 7 slices of the next step, so steps need no cluster barrier.

constexpr int LT_ROWS = 128;                     // gate rows per CTA (32 units x 4 gates)
constexpr int LT_KC = LC_H / 8;                  // 8-element K chunks of the recurrent product
constexpr int LT_ABYTES = LT_KC * LT_ROWS * 16;  // one bf16 W image (64 KB)
constexpr int LT_HROWS = 2 * LC_IPG;             // H image rows: 32 items hi, then 32 items lo
constexpr int LT_BBYTES = LT_KC * LT_HROWS * 16; // one H image (32 KB)
constexpr int LT_GXLD = 17;                      // transpose staging row (floats)
constexpr int LT_SLICE = 4 * LT_HROWS * 16;      // one CTA's 32 units of an H image (4 KB)
constexpr uint32_t LT_IDESC_HL = idesc_f16(LT_ROWS, LT_HROWS);  // Wh x [Hh | Hl]
constexpr uint32_t LT_IDESC_H = idesc_f16(LT_ROWS, LC_IPG);     // Wl x Hh
constexpr float LT_LO_SCALE = 2048.0f;                          // small parts are stored times 2^11
constexpr float LT_LO_INV = 1.0f / 2048.0f;

__host__ __device__ constexpr size_t lt_smem() {
  return 2 * (size_t)LT_ABYTES + 2 * (size_t)LT_BBYTES + sizeof(float) * (8 * 32 * LT_GXLD);
}

// The cell's sigmoid with the hardware exponential and divide (a few ulp of fp32), and tanh x =
// 2 sigma(2x) - 1 (about 1e-7 absolute): on the kernel test the recurrence's h stays within 3.1e-7
// of float64 (the fp32 kernel with expf / tanhf: 1.9e-7), at 15% less time per step.
__device__ __forceinline__ float sigm_fast(float x) { return __fdividef(1.0f, 1.0f + __expf(-x)); }
__device__ __forceinline__ float tanh_fast(float x) { return fmaf(2.0f, sigm_fast(2.0f * x), -1.0f); }
// fp16 bits of x (round to nearest even) and the fp16 bits of its scaled remainder
__device__ __forceinline__ uint32_t f16_bits(float x) { return (uint32_t)__half_as_ushort(__float2half_rn(x)); }
__device__ __forceinline__ uint32_t f16_lo_bits(float x, uint32_t hi) {
  return f16_bits((x - __half2float(__ushort_as_half((unsigned short)hi))) * LT_LO_SCALE);
}

__global__ void __cluster_dims__(LC_CL, 1, 1) __launch_bounds__(256, 1) lstm_tc_kernel(const LstmArgs a) {
  extern __shared__ __align__(1024) uint8_t sm8[];
  uint8_t* Ahi = sm8;
  uint8_t* Alo = Ahi + LT_ABYTES;
  uint8_t* Bb = Alo + LT_ABYTES;                                  // [2 stages] H images
  float* Gx = reinterpret_cast<float*>(Bb + 2 * LT_BBYTES);       // [8 warps][32 lanes][LT_GXLD]
  __shared__ uint64_t bar;
  __shared__ uint64_t hbar[2];  // H image j complete: the 8 CTAs' slices of the next step have landed
  __shared__ uint32_t tslot;
  __shared__ int bad;
  const int rank = (int)cl_rank();
  const int cl = blockIdx.x / LC_CL;
  const int dir = cl & 1, g = cl >> 1;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;

  // W_hh rows of this CTA's units as fp16 hi / scaled-lo operand images (K-major, 8-row x 16-byte cores)
  {
    const float* W = a.whh + (size_t)dir * 4 * LC_H * LC_H;
    for (int idx = tid; idx < LT_ROWS * LC_H; idx += 256) {
      const int ar = idx >> 8, k = idx & 255;
      const int u = rank * 32 + (ar >> 2), gate = ar & 3;
      const float w = W[(size_t)(gate * LC_H + u) * LC_H + k];
      const uint32_t hi = f16_bits(w);
      const uint32_t lo = f16_lo_bits(w, hi);
      const size_t off = (size_t)(k >> 3) * (LT_ROWS * 16) + ar * 16 + (k & 7) * 2;
      *reinterpret_cast<unsigned short*>(Ahi + off) = (unsigned short)hi;
      *reinterpret_cast<unsigned short*>(Alo + off) = (unsigned short)lo;
    }
    for (int i = tid; i < LT_BBYTES / 16; i += 256) reinterpret_cast<uint4*>(Bb)[i] = make_uint4(0, 0, 0, 0);
  }
  // this thread's cells: unit ul (lane quarter q = warp % 4 holds units 8q .. 8q + 7), items i0 .. i0 + 3
  const int q = warp & 3, hf = warp >> 2;
  const int ul = 8 * q + (lane >> 2);
  const int u = rank * 32 + ul;
  const int i0 = hf * 16 + 4 * (lane & 3);
  const int* gs = a.gstart + g * LC_IPG;
  const int* gl = a.glen + g * LC_IPG;
  int st_[4], ln_[4];
#pragma unroll
  for (int m = 0; m < 4; m++) st_[m] = gs[i0 + m], ln_[m] = gl[i0 + m];
  float bh[4];
#pragma unroll
  for (int gt = 0; gt < 4; gt++) bh[gt] = a.bhh[dir * 4 * LC_H + gt * LC_H + u];
  float c[4] = {0.0f, 0.0f, 0.0f, 0.0f};
  const int* act = a.gact + (long)g * a.Tmax;
  // bytes the other 7 CTAs send during step s (into H image (s + 1) & 1): each copies its whole
  // 4 KB slice (rows of finished items are stale and ignored)
  auto push_bytes = [&](int s) -> uint32_t {
    const int n = s + 1 < a.Tmax ? act[s + 1] : 0;
    return n > 0 ? (uint32_t)((LC_CL - 1) * LT_SLICE) : 0u;
  };
  // the cluster addresses of this CTA's slice and of the H-image barriers in each CTA
  uint32_t rblk[LC_CL], rbar0[LC_CL];
  {
    const uint32_t blk = smem_u32(Bb + 4 * rank * (LT_HROWS * 16));
    const uint32_t b0 = smem_u32(&hbar[0]);
#pragma unroll
    for (int r = 0; r < LC_CL; r++) {
      asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(rblk[r]) : "r"(blk), "r"(r));
      asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(rbar0[r]) : "r"(b0), "r"(r));
    }
  }

  if (tid == 0) {
    mbar_init(&bar, 1);
    mbar_init(&hbar[0], 1);
    mbar_init(&hbar[1], 1);
    bad = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    // armed before any CTA can push step 0's results (the cluster barrier below)
    if (push_bytes(0)) mbar_arrive_expect_tx(&hbar[1], push_bytes(0));
  }
  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], 64;" ::"r"(smem_u32(&tslot))
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  fence_proxy_async();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = tslot;
  volatile int abort_flag = 0;
  uint32_t hph[2] = {0, 0};  // phase parity of each H-image barrier
  // gate inputs of this thread's cells for step s (items still running at s), loaded while the
  // step's MMAs run: after the MMA issue, so the issuing thread's proxy fence does not wait on them
  float gxv[4][4];
  auto load_gx = [&](int s, int na) {
#pragma unroll
    for (int m = 0; m < 4; m++) {
#pragma unroll
      for (int gt = 0; gt < 4; gt++) gxv[m][gt] = 0.0f;
      if (i0 + m < na) {
        const int t = dir == 0 ? s : ln_[m] - 1 - s;
        const float* gp = a.gx + (long)(st_[m] + t) * a.ldgx + dir * 4 * LC_H + u;
#pragma unroll
        for (int gt = 0; gt < 4; gt++) gxv[m][gt] = __ldg(gp + gt * LC_H);
      }
    }
  };
  cluster_sync();  // every CTA of the cluster is running and initialised before remote stores

  for (int s = 0; s < a.Tmax; s++) {
    const int na = act[s];
    if (na == 0) break;  // same for the whole group, so for every CTA of the cluster
    const int cur = s & 1;
    // this thread's unit column in this CTA's slice of the next H image (image cur ^ 1)
    uint8_t* hrow = Bb + (cur ^ 1) * LT_BBYTES + (4 * rank + (ul >> 3)) * (LT_HROWS * 16) + (ul & 7) * 2;
    if (s > 0) {  // this step's H image: all 8 CTAs' slices of step s - 1 have landed
      if (!bad && !mbar_wait(&hbar[cur], hph[cur], &abort_flag, a.err)) bad = 1;
      hph[cur] ^= 1;
    }
    if (tid == 0 && !bad) {
      fence_proxy_async();  // the H image arrived through generic-proxy stores
      tc_fence_after();
      // descriptors advance by constant steps of the 14-bit start-address field (16-byte units)
      uint64_t ah = sdesc(smem_u32(Ahi), LT_ROWS * 16, 128);
      uint64_t al = sdesc(smem_u32(Alo), LT_ROWS * 16, 128);
      uint64_t bd = sdesc(smem_u32(Bb + cur * LT_BBYTES), LT_HROWS * 16, 128);
      constexpr uint64_t dA = (2 * LT_ROWS * 16) >> 4, dB = (2 * LT_HROWS * 16) >> 4;
#pragma unroll
      for (int kk = 0; kk < LT_KC / 2; kk++) {
        mma_bf16(tmem, ah, bd, LT_IDESC_HL, kk > 0);       // Wh x [Hh | Hl] -> columns 0..63
        mma_bf16(tmem + LC_IPG, al, bd, LT_IDESC_H, 1);    // Wl x Hh -> columns 32..63
        ah += dA, al += dA, bd += dB;
      }
      mma_commit(&bar);
    }
    load_gx(s, na);
    if (!bad && !mbar_wait(&bar, (uint32_t)(s & 1), &abort_flag, a.err)) bad = 1;
    tc_fence_after();
    __syncthreads();  // bad is uniform from here on
    if (!bad) {
      // lane (unit 8q + lane / 4, gate lane % 4) reads its 16 items of this half (big-part columns
      // and scaled small-part columns), then a 4-lane transpose gives each lane one unit's 4 gates
      // for items i0 .. i0 + 3
      float v[16], w[16];
      tmem_ld16(tmem + ((uint32_t)(q * 32) << 16) + hf * 16, v);
      tmem_ld16(tmem + ((uint32_t)(q * 32) << 16) + LC_IPG + hf * 16, w);
      float* gw = Gx + warp * 32 * LT_GXLD;
#pragma unroll
      for (int j = 0; j < 16; j++) gw[lane * LT_GXLD + j] = fmaf(w[j], LT_LO_INV, v[j]);
      __syncwarp();
      // all four cells are computed unconditionally, so their chains interleave (the cell of an
      // item that has finished, whose gate inputs are zeros, is discarded); only the stores depend
      // on the item still running
      float hv[4];
#pragma unroll
      for (int m = 0; m < 4; m++) {
        float d[4];
#pragma unroll
        for (int gt = 0; gt < 4; gt++) d[gt] = gw[((lane & ~3) + gt) * LT_GXLD + 4 * (lane & 3) + m];
        const float ig = sigm_fast(gxv[m][0] + (d[0] + bh[0]));
        const float fg = sigm_fast(gxv[m][1] + (d[1] + bh[1]));
        const float cg = tanh_fast(gxv[m][2] + (d[2] + bh[2]));
        const float og = sigm_fast(gxv[m][3] + (d[3] + bh[3]));
        c[m] = fg * c[m] + ig * cg;
        hv[m] = og * tanh_fast(c[m]);
      }
#pragma unroll
      for (int m = 0; m < 4; m++) {
        if (i0 + m < na) {
          // the new h goes straight into this CTA's slice of the next H image (fp16 big part in
          // row item, scaled small part in row 32 + item, unit ul's two bytes) and to the output
          const uint32_t hb = f16_bits(hv[m]);
          *reinterpret_cast<unsigned short*>(hrow + (i0 + m) * 16) = (unsigned short)hb;
          *reinterpret_cast<unsigned short*>(hrow + (LC_IPG + i0 + m) * 16) = (unsigned short)f16_lo_bits(hv[m], hb);
          const int t = dir == 0 ? s : ln_[m] - 1 - s;
          a.out[(long)(st_[m] + t) * a.ldo + dir * LC_H + u] = hv[m];
        }
      }
    }
    // re-arm image `cur` (consumed this step) for the pushes of step s + 1, before the barrier that
    // releases this CTA's own step-s pushes: no CTA can push step s + 1 before it has received them
    if (tid == 0 && !bad && push_bytes(s + 1)) mbar_arrive_expect_tx(&hbar[cur], push_bytes(s + 1));
    const int na_next = s + 1 < a.Tmax ? act[s + 1] : 0;
    // this CTA's slice of the next H image is complete: one bulk copy sends it to each other CTA
    // of the cluster, completing bytes of that CTA's barrier for the image
    tc_fence_before();
    fence_proxy_async();
    __syncthreads();  // slice complete; TMEM and staging reads done
    if (tid == 0 && !bad && na_next > 0) {
      const uint32_t src = smem_u32(Bb + (cur ^ 1) * LT_BBYTES + 4 * rank * (LT_HROWS * 16));
      const uint32_t off = (uint32_t)((cur ^ 1) * LT_BBYTES), boff = (uint32_t)((cur ^ 1) * 8);
#pragma unroll
      for (int r = 0; r < LC_CL; r++)
        if (r != rank)
          asm volatile("cp.async.bulk.shared::cluster.shared::cta.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::
                           "r"(rblk[r] + off),
                       "r"(src), "n"(LT_SLICE), "r"(rbar0[r] + boff)
                       : "memory");
    }
  }
  // every push was awaited by its receiver inside the loop; the barrier keeps each CTA (and its
  // shared memory) alive until the whole cluster has left the loop
  cluster_sync();
  if (bad && tid == 0) atomicExch(a.err, 4);
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, 64;" ::"r"(tmem) : "memory");
  }
}

}  // namespace

cudaError_t launch_lstm(const LstmArgs& a, cudaStream_t st) {
  if (a.Tmax == 0 || a.G == 0) return cudaSuccess;
  if (a.IPG != LC_IPG) return cudaErrorInvalidValue;
  if (a.tc) {
    static bool attr_tc[64] = {false};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 64 && !attr_tc[dev]) {
      cudaError_t e = cudaFuncSetAttribute(lstm_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)lt_smem());
      if (e != cudaSuccess) return e;
      attr_tc[dev] = true;
    }
    lstm_tc_kernel<<<dim3(a.G * 2 * LC_CL), dim3(256), lt_smem(), st>>>(a);
    return cudaGetLastError();
  }
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
