// ALBERT self-attention on tcgen05 tensor cores (BF16 precision mode).
//
// Per item and head (src/gpu_batch.rs:429-442: scores = Q K^T per head, softmax(scale * scores) over
// the item's own T tokens, ctx = P V), one CTA of 4 warps handles a tile of 128 query rows:
//  1. Q (128 x 64), K (Tp x 64) and V^T (64 x Tp) of the head are read from the qkv rows (f32, rounded
//     to bf16 here, or bf16 rows the QKV projection already rounded the same way) and stored in the
//     canonical no-swizzle K-major operand layout (Tp = T rounded up to 16, rows past T are zero);
//  2. one elected thread issues S = Q K^T (M 128, N <= 256 per instruction, K 64) into TMEM;
//  3. thread r owns query row r = TMEM lane r: it reads its S row from TMEM twice (row maximum, then
//     p = exp(scale * s - max) in fp32 with the fp32 row sum), and writes P as bf16 over the Q / K
//     buffers, which the finished MMAs no longer need;
//  4. O = P V (M 128, N 64, K Tp) accumulates in TMEM columns 0..63, which held S;
//  5. thread r writes ctx row r = O / sum (fp32).
// Items are launched in length buckets (T <= 128, 256, 512), each with the shared memory and TMEM
// columns its longest item needs, so several short-item CTAs share an SM.
// The two waits on MMA completion are bounded (1 s): on expiry the CTA sets the error flag to 3,
// skips the rest of its work, and still releases its TMEM.
#include <cuda_bf16.h>
#include <stdint.h>
#include <string.h>

#include "kk_launch.h"
#include "kk_tc_ptx.cuh"

namespace kk {

namespace {

constexpr int ATT_D = 64;       // head dimension
constexpr int ATT_HEADS = 12;
constexpr int ATT_QT = 128;     // query rows per CTA (TMEM lanes)
// V^T operand: 16-byte rows of 8 keys, 8 dims per core matrix. The 8-dim groups sit 144 bytes
// apart (128 + 16 of padding, a legal descriptor stride), so eight threads storing the same row of
// eight consecutive groups hit eight different bank groups; a key chunk spans 8 groups.
constexpr int ATT_VSB = 144;
constexpr int ATT_VKC = 8 * ATT_VSB;

__device__ __forceinline__ uint4 pack8_bf16(const float* v) {
  uint4 pk;
  __nv_bfloat162 h0 = __floats2bfloat162_rn(v[0], v[1]);
  __nv_bfloat162 h1 = __floats2bfloat162_rn(v[2], v[3]);
  __nv_bfloat162 h2 = __floats2bfloat162_rn(v[4], v[5]);
  __nv_bfloat162 h3 = __floats2bfloat162_rn(v[6], v[7]);
  memcpy(&pk.x, &h0, 4);
  memcpy(&pk.y, &h1, 4);
  memcpy(&pk.z, &h2, 4);
  memcpy(&pk.w, &h3, 4);
  return pk;
}

template <int TMAX>
__host__ __device__ constexpr int att_preg() {  // bytes of the P region (Q and K live at its start until S is done)
  return TMAX * ATT_QT * 2 > 16384 + TMAX * 16 * 8 ? TMAX * ATT_QT * 2 : 16384 + TMAX * 16 * 8;
}
template <int TMAX>
__host__ __device__ constexpr int att_smem() {
  return att_preg<TMAX>() + (TMAX / 8) * ATT_VKC;
}

// BF: the qkv rows are bf16 (ld in elements); else f32.
template <int TMAX, bool BF>
__global__ void __launch_bounds__(128, 1) attn_tc_kernel(const void* __restrict__ qkv, int ld, const ItemTab* items,
                                                         const int2* work, float* ctx, int ldc, int* err,
                                                         uint8_t* ctx_pre, long ctx_pre_rows) {
  extern __shared__ __align__(1024) uint8_t smem[];
  uint8_t* Qs = smem;                          // [8 dim chunks][128 rows][8] bf16
  uint8_t* Ks = smem + 16384;                  // [8 dim chunks][TMAX keys][8]
  uint8_t* Ps = smem;                          // [TMAX / 8 key chunks][128 rows][8] (after S)
  uint8_t* Vt = smem + att_preg<TMAX>();       // [TMAX / 8 key chunks][8 dim groups, ATT_VSB apart][8 dims][8 keys]
  __shared__ uint64_t bar;
  __shared__ uint32_t tslot;
  __shared__ int bad;

  const int2 wk = work[blockIdx.x];
  const int h = blockIdx.y;
  const ItemTab it = items[wk.x];
  const int T = it.tok_len, q0 = wk.y;
  const int Tp = (T + 15) & ~15;
  const int tid = threadIdx.x, warp = tid >> 5;
  const float* base = (const float*)qkv + (long)it.tok_start * ld + h * ATT_D;
  const unsigned short* baseh = (const unsigned short*)qkv + (long)it.tok_start * ld + h * ATT_D;

  if (tid == 0) {
    mbar_init(&bar, 1);
    bad = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&tslot)),
                 "r"((uint32_t)TMAX)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }

  // ---- operands: Q tile, K, V^T as bf16. Every row's (or task's) loads are issued before any of
  // its stores, so each thread has 16-32 loads in flight instead of waiting on them one chunk at a
  // time (the pass is bound by memory latency). A warp stores 32 consecutive rows of one chunk: no
  // shared-memory bank conflicts.
  auto load_row = [&](int row, int off, float4 (&rv)[16]) {
    const float4* p = reinterpret_cast<const float4*>(base + (long)row * ld + off);
#pragma unroll
    for (int c = 0; c < 16; c++) rv[c] = row < T ? __ldg(p + c) : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
  };
  auto store_row = [&](uint8_t* dst, int stride, int row, const float4 (&rv)[16]) {
#pragma unroll
    for (int c = 0; c < 8; c++) {
      const float v[8] = {rv[2 * c].x, rv[2 * c].y, rv[2 * c].z, rv[2 * c].w,
                          rv[2 * c + 1].x, rv[2 * c + 1].y, rv[2 * c + 1].z, rv[2 * c + 1].w};
      *reinterpret_cast<uint4*>(dst + c * stride + row * 16) = pack8_bf16(v);
    }
  };
  // bf16 rows: 8 dims per 16-byte load, already the operand's 16-byte chunk
  auto copy_row_h = [&](uint8_t* dst, int stride, int row, int drow, int off) {
    const uint4* p = reinterpret_cast<const uint4*>(baseh + (long)row * ld + off);
    uint4 rv[8];
#pragma unroll
    for (int c = 0; c < 8; c++) rv[c] = row < T ? __ldg(p + c) : make_uint4(0u, 0u, 0u, 0u);
#pragma unroll
    for (int c = 0; c < 8; c++) *reinterpret_cast<uint4*>(dst + c * stride + drow * 16) = rv[c];
  };
  if constexpr (BF) {
    copy_row_h(Qs, ATT_QT * 16, q0 + tid, tid, 0);
    for (int j = tid; j < Tp; j += 128) copy_row_h(Ks, TMAX * 16, j, j, 768);
  } else {
    {
      float4 rv[16];
      load_row(q0 + tid, 0, rv);
      store_row(Qs, ATT_QT * 16, tid, rv);
    }
    for (int j = tid; j < Tp; j += 128) {
      float4 rv[16];
      load_row(j, 768, rv);
      store_row(Ks, TMAX * 16, j, rv);
    }
  }
  // V^T: task (key chunk kc, dim d): 8 keys of one dim -> one 16-byte store (a warp covers 32
  // consecutive dims of one key chunk: coalesced loads, conflict-free stores); 4 tasks per thread
  // in flight
  const int ntask = (Tp / 8) * ATT_D;
  if constexpr (BF) {
    // task (key chunk kc, dim group dc): eight 16-byte loads (8 dims of 8 keys; the eight threads of a
    // key chunk read whole 128-byte rows), an 8 x 8 transpose by byte permutes, eight 16-byte
    // stores (8 keys of one dim each)
    const int nt = (Tp / 8) * 8;
#pragma unroll 2
    for (int t = tid; t < nt; t += 128) {
      const int dc = t & 7, kc = t >> 3;
      uint4 in[8];
#pragma unroll
      for (int e = 0; e < 8; e++) {
        const int j = kc * 8 + e;
        in[e] = j < T ? __ldg(reinterpret_cast<const uint4*>(baseh + (long)j * ld + 1536 + dc * 8))
                      : make_uint4(0u, 0u, 0u, 0u);
      }
      uint8_t* dst = Vt + kc * ATT_VKC + dc * ATT_VSB;
      auto wd = [](const uint4& v, int w) { return w == 0 ? v.x : (w == 1 ? v.y : (w == 2 ? v.z : v.w)); };
#pragma unroll
      for (int dd = 0; dd < 8; dd++) {
        const int w = dd >> 1;
        const uint32_t sel = (dd & 1) ? 0x7632u : 0x5410u;  // high or low bf16 of each word
        *reinterpret_cast<uint4*>(dst + dd * 16) =
            make_uint4(__byte_perm(wd(in[0], w), wd(in[1], w), sel), __byte_perm(wd(in[2], w), wd(in[3], w), sel),
                       __byte_perm(wd(in[4], w), wd(in[5], w), sel), __byte_perm(wd(in[6], w), wd(in[7], w), sel));
      }
    }
  }
  for (int t0 = 0; !BF && t0 < ntask; t0 += 4 * 128) {
    float v[4][8];
#pragma unroll
    for (int u = 0; u < 4; u++) {
      const int t = t0 + u * 128 + tid, kc = t / ATT_D, d = t % ATT_D;
#pragma unroll
      for (int e = 0; e < 8; e++) {
        const int j = kc * 8 + e;
        v[u][e] = (t < ntask && j < T) ? __ldg(base + (long)j * ld + 1536 + d) : 0.0f;
      }
    }
#pragma unroll
    for (int u = 0; u < 4; u++) {
      const int t = t0 + u * 128 + tid, kc = t / ATT_D, d = t % ATT_D;
      if (t < ntask)
        *reinterpret_cast<uint4*>(Vt + kc * ATT_VKC + (d >> 3) * ATT_VSB + (d & 7) * 16) = pack8_bf16(v[u]);
    }
  }
  fence_proxy_async();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = tslot;

  // ---- S = Q K^T
  if (tid == 0) {
    for (int g = 0; g * 256 < Tp; g++) {
      const int ng = Tp - g * 256 < 256 ? Tp - g * 256 : 256;
      const uint32_t id = idesc_bf16(ATT_QT, ng);
#pragma unroll
      for (int kk = 0; kk < ATT_D / 16; kk++) {
        const uint64_t ad = sdesc(smem_u32(Qs) + kk * 2 * (ATT_QT * 16), ATT_QT * 16, 128);
        const uint64_t bd = sdesc(smem_u32(Ks) + kk * 2 * (TMAX * 16) + g * 256 * 16, TMAX * 16, 128);
        mma_bf16(tmem + g * 256, ad, bd, id, kk > 0);
      }
    }
    mma_commit(&bar);
  }
  volatile int abort_flag = 0;
  if (!mbar_wait(&bar, 0, &abort_flag, err)) bad = 1;
  tc_fence_after();
  __syncthreads();

  // ---- softmax of row r (TMEM lane r; warp w reads lanes 32w .. 32w + 31)
  const uint32_t trow = tmem + ((uint32_t)(warp * 32) << 16);
  float l = 0.0f;
  if (!bad) {
    const float scale = 0.125f;  // head_dim^-0.5
    float m = -INFINITY;
    for (int c0 = 0; c0 < Tp; c0 += 32) {
      float s[32];
      tmem_ld32(trow + c0, s);
#pragma unroll
      for (int e = 0; e < 32; e++)
        if (c0 + e < T) m = fmaxf(m, s[e] * scale);
    }
    for (int c0 = 0; c0 < Tp; c0 += 32) {
      float s[32];
      tmem_ld32(trow + c0, s);
#pragma unroll
      for (int e = 0; e < 32; e++) {
        const float pv = c0 + e < T ? expf(s[e] * scale - m) : 0.0f;
        l += pv;
        s[e] = pv;
      }
#pragma unroll
      for (int e = 0; e < 32; e += 8)
        if (c0 + e < Tp) *reinterpret_cast<uint4*>(Ps + ((c0 + e) >> 3) * (ATT_QT * 16) + tid * 16) = pack8_bf16(s + e);
    }
  }
  fence_proxy_async();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();

  // ---- O = P V into TMEM columns 0..63
  if (tid == 0 && !bad) {
    const uint32_t id = idesc_bf16(ATT_QT, ATT_D);
    for (int kk = 0; kk < Tp / 16; kk++) {
      const uint64_t ad = sdesc(smem_u32(Ps) + kk * 2 * (ATT_QT * 16), ATT_QT * 16, 128);
      const uint64_t bd = sdesc(smem_u32(Vt) + kk * 2 * ATT_VKC, ATT_VKC, ATT_VSB);
      mma_bf16(tmem, ad, bd, id, kk > 0);
    }
    mma_commit(&bar);
  }
  if (!bad && !mbar_wait(&bar, 1, &abort_flag, err)) bad = 1;
  tc_fence_after();
  __syncthreads();

  // ---- ctx row = O / sum. tcgen05.ld is warp-collective (.sync.aligned): every lane loads, only
  // the rows of real queries are stored. `bad` is uniform here (read after the barrier).
  if (!bad) {
    const float inv = 1.0f / l;
    const bool row_ok = q0 + tid < T;
    const long row = it.tok_start + q0 + tid;
    float* out = ctx + row * ldc + h * ATT_D;
#pragma unroll
    for (int c0 = 0; c0 < ATT_D; c0 += 32) {
      float o[32];
      tmem_ld32(trow + c0, o);
      if (row_ok && ctx_pre) {
        // head h is 64-channel block h of the planes: channels c0 + 4j .. + 3 are half c0 / 32 of
        // chunk j
#pragma unroll
        for (int jc = 0; jc < 8; jc++) {
          __nv_bfloat162 p0 = __floats2bfloat162_rn(o[4 * jc] * inv, o[4 * jc + 1] * inv);
          __nv_bfloat162 p1 = __floats2bfloat162_rn(o[4 * jc + 2] * inv, o[4 * jc + 3] * inv);
          uint2 u;
          memcpy(&u.x, &p0, 4);
          memcpy(&u.y, &p1, 4);
          *reinterpret_cast<uint2*>(ctx_pre + ((size_t)(h * 8 + jc) * ctx_pre_rows + PRE_PAD_FRONT + row) * 16 +
                                    (c0 >> 5) * 8) = u;
        }
      } else if (row_ok) {
#pragma unroll
        for (int e = 0; e < 32; e += 4)
          *reinterpret_cast<float4*>(out + c0 + e) =
              make_float4(o[e] * inv, o[e + 1] * inv, o[e + 2] * inv, o[e + 3] * inv);
      }
    }
  }
  if (bad && tid == 0) atomicExch(err, 3);
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"((uint32_t)TMAX) : "memory");
  }
}

template <int TMAX, bool BF>
cudaError_t launch_bucket(const void* qkv, int ld, const ItemTab* items, const int2* work, int n, float* ctx, int ldc,
                          int* err, cudaStream_t st, void* ctx_pre, long ctx_pre_rows) {
  if (n == 0) return cudaSuccess;
  static bool attr[64] = {false};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 64 && !attr[dev]) {
    cudaError_t e = cudaFuncSetAttribute(attn_tc_kernel<TMAX, BF>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         att_smem<TMAX>());
    if (e != cudaSuccess) return e;
    attr[dev] = true;
  }
  attn_tc_kernel<TMAX, BF><<<dim3(n, ATT_HEADS), 128, att_smem<TMAX>(), st>>>(qkv, ld, items, work, ctx, ldc, err,
                                                                               (uint8_t*)ctx_pre, ctx_pre_rows);
  return cudaGetLastError();
}

template <bool BF>
cudaError_t launch_buckets(const void* qkv, int ldqkv, const ItemTab* items, const int2* work, const int n_work[3],
                           float* ctx, int ldc, int* err, cudaStream_t st, void* ctx_pre, long ctx_pre_rows) {
  cudaError_t e = launch_bucket<128, BF>(qkv, ldqkv, items, work, n_work[0], ctx, ldc, err, st, ctx_pre, ctx_pre_rows);
  if (e == cudaSuccess)
    e = launch_bucket<256, BF>(qkv, ldqkv, items, work + n_work[0], n_work[1], ctx, ldc, err, st, ctx_pre,
                               ctx_pre_rows);
  if (e == cudaSuccess)
    e = launch_bucket<512, BF>(qkv, ldqkv, items, work + n_work[0] + n_work[1], n_work[2], ctx, ldc, err, st, ctx_pre,
                               ctx_pre_rows);
  return e;
}

}  // namespace

cudaError_t launch_attention_tc(const void* qkv, int ldqkv, bool qkv_bf16, const ItemTab* items, const int2* work,
                                const int n_work[3], float* ctx, int ldc, int* err, cudaStream_t st, void* ctx_pre,
                                long ctx_pre_rows) {
  if (ctx_pre && (((uintptr_t)ctx_pre) & 15) != 0) return cudaErrorInvalidValue;
  // 16-byte row loads: bf16 rows need a 16-byte aligned base and a row stride of 8 elements
  if (qkv_bf16 && ((((uintptr_t)qkv) & 15) != 0 || ldqkv % 8 != 0)) return cudaErrorInvalidValue;
  return qkv_bf16 ? launch_buckets<true>(qkv, ldqkv, items, work, n_work, ctx, ldc, err, st, ctx_pre, ctx_pre_rows)
                  : launch_buckets<false>(qkv, ldqkv, items, work, n_work, ctx, ldc, err, st, ctx_pre, ctx_pre_rows);
}

}  // namespace kk
