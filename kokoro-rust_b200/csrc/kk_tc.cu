// tcgen05 implicit-GEMM 1-D convolution (BF16 precision mode).
//
// GEMM view of one output tile: D[co, t] (TMEM, fp32, 128 lanes x 256 columns) =
//   sum over input-channel blocks cb (64 channels) and taps k of
//   A_k,cb[co, ci] (weights, bf16, K-major)  x  B_k,cb[t, ci] (activations, bf16, K-major)
// issued as tcgen05.mma.cta_group::1.kind::f16 with M = 128, N = 256, K = 16.
//
// Operand staging (canonical no-swizzle K-major layout of 8-row x 16-byte core matrices):
//  * weights: a load-time image of 16 KB blocks [co tile][cb][tap], each block laid out exactly as
//    its shared-memory operand (LBO 2048 B between 8-channel chunks, SBO 128 B between 8-row
//    groups), streamed with one cp.async.bulk per block into a 3-stage ring;
//  * input rows: a loader warp streams the f32 rows of each tile's window
//    [t0 - pad, t0 + 256 + (K-1)*dil - pad) with TMA tensor loads (boxes of 64 channels x 32 rows,
//    8 KB, or 64 rows, 16 KB, for layers without a residual read; rows and channels outside the
//    tensor read as zero) into a ring of up to 6 stages, so
//    HBM latency is covered by the ring depth rather than by registers;
//  * activations: 4 producer warps read the boxes from shared memory, apply the layer's prologue
//    (gap masking, AdaIN + leaky ReLU, AdaIN + Snake, leaky ReLU, nearest x2 upsample) and store
//    bf16 in a time-contiguous layout: chunk j (8 channels) holds all window rows at 16 B per row.
//    Because the rows of a chunk are contiguous, the B operand of tap k is the same window with its
//    start address moved by k * dil rows: the window is staged once per channel block and reused by
//    every tap (implicit GEMM; no im2col, no per-tap reload). Within a 64-channel block, chunk j
//    holds channels 4j..4j+3 and 32+4j..32+4j+3 (the weight image uses the same order), so the 8
//    lanes that convert one box row read 128 contiguous bytes (no bank conflicts);
//  * accumulators: two 256-column TMEM buffers, so the epilogue of one tile overlaps the MMAs of
//    the next. 8 epilogue warps (two per TMEM lane quarter, each owning 128 of the tile's 256 time
//    rows) apply bias / residual / shortcut / gelu and the fused AdaIN statistics, stage 16-row x
//    32-channel boxes in shared memory and write them with TMA tensor stores; residual rows arrive
//    by TMA tensor loads two boxes ahead.
//
// Warp roles (20 warps): 0 weight loader + TMEM owner, 1 MMA issuer (one elected lane), 2 input
// loader, 3 row items and coefficient tables (fused route), 4-11 epilogue, 12-19 activation
// producers. Persistent CTAs walk the tiles in output-channel-fastest order: the CTAs running
// together cover every co tile of a few time tiles, so each input window leaves HBM once and the
// other co tiles read it from L2 (a layer's weights, at most a few MB, stay in L2 throughout).
//
// Every mbarrier wait is bounded (1 s of %globaltimer): on expiry the CTA records the failure in
// the engine's error flag, drains its own bulk copies (bounded), releases its TMEM and returns.
#include <cuda.h>
#include <cuda_bf16.h>
#include <stdint.h>
#include <string.h>
#include <vector>

#include "kk_tc.h"
#include "kk_tc_ptx.cuh"

namespace kk {

constexpr int TC_M = 128;
constexpr int TC_N = 256;
constexpr int TC_KB = 64;
constexpr int TC_WST = 3;                        // weight ring stages
constexpr int TC_XST_MAX = 4;                    // activation-window stages (2 on the fused route)
constexpr int TC_RST_MAX = 6;                    // input-box ring stages (fewer when shared memory is short)
constexpr int TC_BOX_ROWS = 32;                  // input box rows (64 for stores without a residual read)
// Input box rows of an instance: 64 (16 KB boxes, each producer thread converts two rows per box
// wait) when the epilogue reads no residual; 32 otherwise, where the residual buffers leave room
// for a deeper ring of smaller boxes only.
__host__ __device__ constexpr int tc_box_rows(int im, int om) {
  return (im >= 0 && im != IN_PRE && (om == OUT_STORE || om == OUT_GELU)) ? 64 : TC_BOX_ROWS;
}
constexpr int TC_MAX_WIN = 512;
constexpr int TC_EC = 16;                        // epilogue chunk: 16 time rows x 32 channels per warp
constexpr int TC_RES_DEPTH = 2;                  // residual chunks in flight per epilogue warp
constexpr int TC_EBOX = TC_EC * 32 * 4;          // 2 KB: one warp's chunk (TMA box 32 channels x 16 rows)
constexpr int TC_NEPI = 8;                       // epilogue warps
constexpr int TC_NPROD = 8;                      // producer warps
constexpr int TC_PROWS = TC_NPROD * 32 / 8;      // box rows converted at once (8 lanes per row)
constexpr int TC_EROWS = TC_N / 2;               // time rows per epilogue warp
// per epilogue warp: 2 staging chunks, TC_RES_DEPTH residual chunks (only for residual / shortcut
// epilogues), the item of each output row
__host__ __device__ constexpr int tc_epi_warp_bytes(bool need_res) {
  return (2 + (need_res ? TC_RES_DEPTH : 0)) * TC_EBOX + TC_EROWS * 4;
}
constexpr int TC_TAB = 256;                      // channels of the shared-memory coefficient tables
constexpr int TC_THREADS = (4 + TC_NEPI + TC_NPROD) * 32;
constexpr int TC_WBLOCK = TC_M * TC_KB * 2;      // 16 KB weight block
constexpr int TC_SMEM_MAX = 227 * 1024;
constexpr unsigned long long TC_TIMEOUT_NS = KK_WAIT_TIMEOUT_NS;
constexpr uint32_t TC_IDESC = idesc_bf16(TC_M, TC_N);

// ------------------------------------------------------------------------------ kernel

struct TcArgs {
  CUtensorMap xmap;   // input rows [L_x][cin] f32 (row stride ldx), box 64 channels x 32 rows
  CUtensorMap ymap;   // output rows [L_out][cout] f32 (row stride ldy), box 32 channels x 16 rows
  CUtensorMap rmap;   // residual rows (y for OUT_ADD, sc for OUT_PLUS), same box
  ConvArgs a;
  const __nv_bfloat16* wimg;
  int ncb;        // input-channel blocks of 64
  int n_cot;      // output-channel tiles of 128
  int n_tt;       // time tiles of 256
  int win_rows;   // 256 + (K - 1) * dil
  int win_pad;    // window rows rounded to 8, + 1 (bank-conflict-free producer stores)
  int rst;        // input-box ring stages (0 on the pre-transform route)
  int xst;        // activation-window stages
  int red;        // OUT_ADD without statistics: the TMA unit adds the staged result into y
  int epb;        // shared-memory bytes per epilogue warp
  int tab;        // AdaIN coefficients and Snake alphas come from shared-memory tables (cin <= TC_TAB)
  int* err;
  unsigned long long* trace;  // optional cycle accounting of CTA 0 (diagnostics), 16 counters
};

// Cycle accounting (CTA 0, when p.trace is set): slot indices.
enum TcTrace : int {
  TR_MMA_WAIT_ACC = 0, TR_MMA_WAIT_X = 1, TR_MMA_WAIT_W = 2, TR_MMA_TOTAL = 3,
  TR_LD_WAIT_W = 4, TR_LD_TOTAL = 5,
  TR_PR_WAIT_X = 6, TR_PR_WORK = 7, TR_PR_WAIT_IN = 8,
  TR_EP_WAIT = 9, TR_EP_WORK = 10, TR_TILES = 11,
  TR_IN_WAIT = 12, TR_IN_TOTAL = 13, TR_EP_RES = 14, TR_EP_STBUF = 15
};

// First and last input row (of the tensor x) of a tile's window, and the number of input boxes.
struct InSpan {
  int base, xr0, nbox;
};
__device__ __forceinline__ InSpan in_span(const TcArgs& p, int tile, int up2, int box_rows) {
  InSpan s;
  s.base = (tile / p.n_cot) * TC_N - p.a.pad;
  const int last = s.base + p.win_rows - 1;
  s.xr0 = up2 ? (s.base >> 1) : s.base;
  const int xr1 = up2 ? (last >> 1) : last;
  s.nbox = (xr1 - s.xr0) / box_rows + 1;
  return s;
}

// IM / UP / OM: the layer's input mode, nearest x2 upsample and output mode as compile-time
// constants (branch-free producer and epilogue loops); IM = -1 is the generic instance that reads
// all three from the arguments.
template <int IM, int UP, int OM>
__global__ void __launch_bounds__(TC_THREADS, 1) tc_conv_kernel(const __grid_constant__ TcArgs p) {
  extern __shared__ __align__(1024) uint8_t smem[];
  const ConvArgs& a = p.a;
  const int in_mode = IM >= 0 ? IM : a.in_mode;
  const int in_up2 = IM >= 0 ? UP : a.in_up2;
  // OUT_STORE_BF runs as OUT_STORE with bf16 staging and a bf16 tensor map
  constexpr bool YB = OM == OUT_STORE_BF;
  const int out_mode_k = IM >= 0 ? (YB ? OUT_STORE : OM) : a.out_mode;
  const uint32_t xbytes = 8u * p.win_pad * 16u;
  const int RST = p.rst;
  constexpr int BOXR = tc_box_rows(IM, OM);
  constexpr uint32_t INBOX = BOXR * TC_KB * 4;
  uint8_t* wbuf = smem;                                       // TC_WST x 16 KB
  const int XST = p.xst;
  uint8_t* xbuf = wbuf + TC_WST * TC_WBLOCK;                  // XST x xbytes
  uint8_t* inring = xbuf + XST * xbytes;                      // RST x 8 KB
  uint8_t* epi = inring + RST * INBOX;                        // TC_NEPI x p.epb
  uint64_t* bars = (uint64_t*)(epi + TC_NEPI * p.epb);
  uint64_t* w_full = bars;
  uint64_t* w_empty = w_full + TC_WST;
  uint64_t* in_full = w_empty + TC_WST;
  uint64_t* in_empty = in_full + TC_RST_MAX;
  uint64_t* x_full = in_empty + TC_RST_MAX;
  uint64_t* x_empty = x_full + TC_XST_MAX;
  uint64_t* acc_full = x_empty + TC_XST_MAX;
  uint64_t* acc_empty = acc_full + 2;
  uint64_t* res_full = acc_empty + 2;                         // [TC_NEPI][TC_RES_DEPTH]
  uint64_t* meta_full = res_full + TC_NEPI * TC_RES_DEPTH;    // [2] a tile's row items / coefficients written
  uint64_t* meta_empty = meta_full + 2;                       // [2] the producers are done with them
  uint32_t* tmem_slot = (uint32_t*)(meta_empty + 2);
  volatile int* abort_flag = (volatile int*)(tmem_slot + 1);
  int* mitem = (int*)(tmem_slot + 2);                         // [2] item whose coefficients ctab holds
  int* ritem = (int*)(tmem_slot + 4);                         // [2][TC_MAX_WIN] item of each window row
  // The coefficient tables are pair-interleaved: channels 2i and 2i + 1 as one float4 {scale0, scale1,
  // shift0, shift1} ({alpha0, alpha1, 1 / alpha0, 1 / alpha1}), so a producer's 16-byte load yields the
  // register pairs its packed f32x2 arithmetic takes.
  float* ctab = (float*)(ritem + 2 * TC_MAX_WIN);             // [2][TC_TAB] AdaIN (scale, shift) of mitem
  float* atab = ctab + 2 * 2 * TC_TAB;                        // [TC_TAB] Snake (alpha, 1 / alpha)

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int ntiles = p.n_cot * p.n_tt;
  const int K = a.K;

  if (threadIdx.x == 0) {
    for (int i = 0; i < TC_WST; i++) {
      mbar_init(&w_full[i], 1);
      mbar_init(&w_empty[i], 1);
    }
    for (int i = 0; i < RST; i++) {
      mbar_init(&in_full[i], 1);
      mbar_init(&in_empty[i], TC_NPROD);
    }
    for (int i = 0; i < XST; i++) {
      mbar_init(&x_full[i], IM == IN_PRE ? 1 : TC_NPROD);  // IN_PRE: the loader's expect_tx arrival
      mbar_init(&x_empty[i], 1);
    }
    for (int i = 0; i < 2; i++) {
      mbar_init(&acc_full[i], 1);
      mbar_init(&acc_empty[i], TC_NEPI);
    }
    for (int i = 0; i < TC_NEPI * TC_RES_DEPTH; i++) mbar_init(&res_full[i], 1);
    for (int i = 0; i < 2; i++) {
      mbar_init(&meta_full[i], 1);
      mbar_init(&meta_empty[i], TC_NPROD);
    }
    *abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], 512;" ::"r"(smem_u32(tmem_slot))
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    // ---------------------------------------------------------------- weight loader
    if (lane == 0) {
      unsigned long long tw = 0;
      unsigned long long* tr = (p.trace && blockIdx.x == 0) ? &tw : nullptr;
      const long long t_start = clock64();
      uint32_t it = 0;
      for (int tile = blockIdx.x; tile < ntiles && !*abort_flag; tile += gridDim.x) {
        const int cot = tile % p.n_cot;
        const uint8_t* src = (const uint8_t*)p.wimg + (size_t)cot * p.ncb * K * TC_WBLOCK;
        for (int s = 0; s < p.ncb * K; s++, it++) {
          const int st = it % TC_WST;
          if (!mbar_wait_t(&w_empty[st], ((it / TC_WST) & 1) ^ 1, abort_flag, p.err, tr)) break;
          mbar_arrive_expect_tx(&w_full[st], TC_WBLOCK);
          bulk_g2s(wbuf + st * TC_WBLOCK, src + (size_t)s * TC_WBLOCK, TC_WBLOCK, &w_full[st]);
        }
      }
      if (tr) {
        p.trace[TR_LD_WAIT_W] = tw;
        p.trace[TR_LD_TOTAL] = (unsigned long long)(clock64() - t_start);
      }
      if (*abort_flag) {
        // drain this CTA's bulk copies still in flight before the shared memory is released
        const uint32_t first = it > TC_WST ? it - TC_WST : 0;
        for (uint32_t j = first; j < it; j++) {
          const unsigned long long t0 = tc_now();
          while (!mbar_try(&w_full[j % TC_WST], (j / TC_WST) & 1) && tc_now() - t0 < TC_TIMEOUT_NS) {
          }
        }
      }
    }
  } else if (warp == 1) {
    // ---------------------------------------------------------------- MMA issuer
    if (lane == 0) {
      unsigned long long twa = 0, twx = 0, tww = 0;
      const bool trc = p.trace && blockIdx.x == 0;
      const long long t_start = clock64();
      uint32_t wit = 0, xit = 0, lt = 0;
      for (int tile = blockIdx.x; tile < ntiles; tile += gridDim.x, lt++) {
        const int ab = lt & 1;
        if (!mbar_wait_t(&acc_empty[ab], ((lt >> 1) & 1) ^ 1, abort_flag, p.err, trc ? &twa : nullptr)) break;
        tc_fence_after();
        const uint32_t d = tmem + ab * TC_N;
        bool ok = true;
        for (int cb = 0; cb < p.ncb && ok; cb++, xit++) {
          const int xs = xit % XST;
          if (!mbar_wait_t(&x_full[xs], (xit / XST) & 1, abort_flag, p.err, trc ? &twx : nullptr)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t xb = smem_u32(xbuf + xs * xbytes);
          for (int k = 0; k < K; k++, wit++) {
            const int ws = wit % TC_WST;
            if (!mbar_wait_t(&w_full[ws], (wit / TC_WST) & 1, abort_flag, p.err, trc ? &tww : nullptr)) {
              ok = false;
              break;
            }
            tc_fence_after();
            const uint32_t wb = smem_u32(wbuf + ws * TC_WBLOCK);
#pragma unroll
            for (int kk = 0; kk < 4; kk++) {
              const uint64_t ad = sdesc(wb + kk * 2 * 2048, 2048, 128);
              const uint64_t bd = sdesc(xb + (uint32_t)(k * a.dil) * 16u + kk * 2 * 16u * p.win_pad,
                                        16u * p.win_pad, 128);
              mma_bf16(d, ad, bd, TC_IDESC, (cb | k | kk) != 0);
            }
            mma_commit(&w_empty[ws]);
          }
          if (ok) mma_commit(&x_empty[xs]);
        }
        if (!ok) break;
        mma_commit(&acc_full[ab]);
      }
      if (trc) {
        p.trace[TR_MMA_WAIT_ACC] = twa;
        p.trace[TR_MMA_WAIT_X] = twx;
        p.trace[TR_MMA_WAIT_W] = tww;
        p.trace[TR_MMA_TOTAL] = (unsigned long long)(clock64() - t_start);
        p.trace[TR_TILES] = lt;
      }
    }
  } else if (warp == 2 && IM == IN_PRE) {
    // ---------------------------------------------------------------- window loader (IN_PRE)
    // Each window chunk is a contiguous run of win_rows 16-byte plane rows: one bulk copy per
    // chunk, straight into the MMA operand layout.
    if (lane == 0) {
      const uint8_t* planes = (const uint8_t*)a.xpre;
      uint32_t xit = 0;
      bool ok = true;
      for (int tile = blockIdx.x; tile < ntiles && ok; tile += gridDim.x) {
        const long row0 = (long)(tile / p.n_cot) * TC_N - a.pad + PRE_PAD_FRONT;
        for (int cb = 0; cb < p.ncb; cb++, xit++) {
          const int xs = xit % XST;
          if (!mbar_wait(&x_empty[xs], ((xit / XST) & 1) ^ 1, abort_flag, p.err)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(&x_full[xs], 8u * p.win_rows * 16u);
          for (int j = 0; j < 8; j++)
            bulk_g2s(xbuf + xs * xbytes + (size_t)j * 16 * p.win_pad,
                     planes + ((size_t)(cb * 8 + j) * a.pre_rows + row0) * 16, (uint32_t)p.win_rows * 16u,
                     &x_full[xs]);
        }
      }
      if (*abort_flag && xit > 0) {
        // drain this CTA's copies still in flight before the shared memory is released
        const uint32_t first = xit > (uint32_t)XST ? xit - XST : 0;
        for (uint32_t jx = first; jx < xit; jx++) {
          const unsigned long long t0 = tc_now();
          while (!mbar_try(&x_full[jx % XST], (jx / XST) & 1) && tc_now() - t0 < TC_TIMEOUT_NS) {
          }
        }
      }
    }
  } else if (warp == 2) {
    // ---------------------------------------------------------------- input loader
    if (lane == 0) {
      unsigned long long tw = 0;
      unsigned long long* tr = (p.trace && blockIdx.x == 0) ? &tw : nullptr;
      const long long t_start = clock64();
      uint32_t it = 0;
      int sl = 0;
      uint32_t ph = 0;  // ring slot and phase parity of box `it`
      bool ok = true;
      for (int tile = blockIdx.x; tile < ntiles && ok; tile += gridDim.x) {
        const InSpan sp = in_span(p, tile, in_up2, BOXR);
        for (int cb = 0; cb < p.ncb && ok; cb++)
          for (int i = 0; i < sp.nbox; i++, it++) {
            if (!mbar_wait_t(&in_empty[sl], ph ^ 1, abort_flag, p.err, tr)) {
              ok = false;
              break;
            }
            mbar_arrive_expect_tx(&in_full[sl], INBOX);
            tma_load_2d(inring + sl * INBOX, &p.xmap, cb * TC_KB, sp.xr0 + i * BOXR, &in_full[sl]);
            if (++sl == RST) sl = 0, ph ^= 1;
          }
      }
      if (tr) {
        p.trace[TR_IN_WAIT] = tw;
        p.trace[TR_IN_TOTAL] = (unsigned long long)(clock64() - t_start);
      }
      if (*abort_flag) {
        const uint32_t first = it > (uint32_t)RST ? it - RST : 0;
        for (uint32_t j = first; j < it; j++) {
          const unsigned long long t0 = tc_now();
          while (!mbar_try(&in_full[j % RST], (j / RST) & 1) && tc_now() - t0 < TC_TIMEOUT_NS) {
          }
        }
      }
    }
  } else if (warp == 3 && IM != IN_PRE) {
    // ---------------------------------------------------------------- row items and coefficients
    // One tile ahead of the producers, this warp writes into the tile's half of the double-buffered
    // tables the item of every window row and, when the prologue is affine and cin <= TC_TAB, the
    // AdaIN (scale, shift) of one item of the window (that of its middle row; items span
    // thousands of rows, so it is nearly always every row's) for all channels; the Snake
    // (alpha, 1 / alpha) table is written once, before the first tile. The producers then read
    // shared memory where they would otherwise wait on global loads at every tile and channel
    // block. All loads of a table are issued before any is stored.
    const int cin = a.cin, win_rows = p.win_rows;
    const bool tab = p.tab != 0;
    if (tab && in_mode == IN_ADAIN_SNAKE) {
      float av[TC_TAB / 32];
#pragma unroll
      for (int k = 0; k < TC_TAB / 32; k++) {
        const int c = lane + 32 * k;
        av[k] = c < cin ? a.alpha[c] : 1.0f;
      }
#pragma unroll
      for (int k = 0; k < TC_TAB / 32; k++) {
        const int c = lane + 32 * k;
        atab[(c >> 1) * 4 + (c & 1)] = av[k];
        atab[(c >> 1) * 4 + 2 + (c & 1)] = 1.0f / av[k];
      }
    }
    uint32_t lt = 0;
    for (int tile = blockIdx.x; tile < ntiles; tile += gridDim.x, lt++) {
      const int bf = lt & 1;
      if (!mbar_wait(&meta_empty[bf], ((lt >> 1) & 1) ^ 1, abort_flag, p.err)) break;
      const InSpan sp = in_span(p, tile, in_up2, BOXR);
      int* ri = ritem + bf * TC_MAX_WIN;
      int iv[TC_MAX_WIN / 32];
#pragma unroll
      for (int k = 0; k < TC_MAX_WIN / 32; k++) {
        const int r = lane + 32 * k, g = sp.base + r;
        iv[k] = (r >= win_rows || g < 0 || g >= a.L_in) ? -1 : (in_mode == IN_NOMASK ? 0 : dom_item(a.din, g));
      }
#pragma unroll
      for (int k = 0; k < TC_MAX_WIN / 32; k++)
        if (lane + 32 * k < win_rows) ri[lane + 32 * k] = iv[k];
      __syncwarp();
      if (tab) {
        int item = ri[win_rows / 2];
        if (item < 0) item = ri[0] >= 0 ? ri[0] : ri[win_rows - 1];
        float2 cv[TC_TAB / 32];
#pragma unroll
        for (int k = 0; k < TC_TAB / 32; k++) {
          const int c = lane + 32 * k;
          cv[k] = (item >= 0 && c < cin) ? a.coef[(long)item * cin + c] : make_float2(0.0f, 0.0f);
        }
        float* ct = ctab + bf * 2 * TC_TAB;
#pragma unroll
        for (int k = 0; k < TC_TAB / 32; k++) {
          const int c = lane + 32 * k;
          ct[(c >> 1) * 4 + (c & 1)] = cv[k].x;
          ct[(c >> 1) * 4 + 2 + (c & 1)] = cv[k].y;
        }
        if (lane == 0) mitem[bf] = item;
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&meta_full[bf]);  // release: the tables are visible to the waiters
    }
  } else if (warp >= 4 && warp < 4 + TC_NEPI) {
    // ---------------------------------------------------------------- epilogue
    // Warp ew owns the 32 channels of TMEM lane quarter q = warp % 4 for time rows
    // [hrow, hrow + 128) of each tile, end to end: its own staging chunks, TMA store boxes
    // (32 channels x 16 rows), residual ring and row-item table, so the warps never wait for one
    // another. When all 128 rows belong to one item (the common case: items span thousands of
    // rows in the frame domains) the statistics accumulate in registers for the whole tile.
    const int ew = warp - 4;
    const int q = warp & 3;
    const int hrow = (ew >> 2) * TC_EROWS;
    // OUT_ADD without statistics needs no residual rows here: the staged acc + bias is added into
    // y by a TMA reduce (the same single f32 addition, done in L2)
    const bool red = out_mode_k == OUT_ADD && p.red;
    const bool need_res = (out_mode_k == OUT_ADD && !red) || out_mode_k == OUT_PLUS;
    float* stg = (float*)(epi + ew * p.epb);                      // [2][16][32]
    float* rsb = stg + 2 * TC_EC * 32;                            // [TC_RES_DEPTH][16][32] (need_res)
    int* eit = (int*)(rsb + (need_res ? TC_RES_DEPTH : 0) * TC_EC * 32);  // [128]
    uint64_t* rbar = res_full + ew * TC_RES_DEPTH;
    constexpr int NCH = TC_EROWS / TC_EC;
    const bool trc = p.trace && blockIdx.x == 0 && ew == 0 && lane == 0;
    unsigned long long tew = 0;
    long long t_res = 0, t_stbuf = 0;
    const long long t_start = clock64();
    uint32_t rcons = 0, riss = 0;  // residual chunks consumed / issued by this warp
    const int out_mode = out_mode_k, L_out = a.L_out;
    const float oscale = a.oscale;
    double* const stat = a.stat;
    uint32_t lt = 0;
    bool bad = false;
    // Items of the first (lane 0) and last (lane 1) of a tile's 128 rows, loaded one tile ahead so
    // the item-table latency hides behind the previous tile's work. Equal ends mean one item
    // covers all 128 rows (item spans are contiguous runs); only tiles that straddle an item
    // boundary or the end build the per-row table.
    auto edge_item = [&](int tl) {
      const int r = (tl / p.n_cot) * TC_N + hrow + (lane == 0 ? 0 : TC_EROWS - 1);
      return (stat && lane < 2 && tl < ntiles && r < L_out) ? dom_item(a.dout, r) : -1;
    };
    int edge_next = edge_item(blockIdx.x);
    for (int tile = blockIdx.x; tile < ntiles && !bad; tile += gridDim.x, lt++) {
      const int ab = lt & 1;
      const int cot = tile % p.n_cot, tt = tile / p.n_cot;
      const int edge = edge_next;
      edge_next = edge_item(tile + gridDim.x);
      const int co0 = cot * TC_M + q * 32;
      const int co = co0 + lane;
      const int t0 = tt * TC_N + hrow;
      const bool co_ok = co < a.cout;
      const float bias = (co_ok && a.bias) ? a.bias[co] : 0.0f;
      // residual chunks of this tile start loading before the accumulator is ready
      if (need_res && lane == 0) {
        for (int c = 0; c < TC_RES_DEPTH; c++, riss++) {
          const int sl = riss % TC_RES_DEPTH;
          mbar_arrive_expect_tx(&rbar[sl], TC_EBOX);
          tma_load_2d(rsb + sl * TC_EC * 32, &p.rmap, co0, t0 + c * TC_EC, &rbar[sl]);
        }
      }
      int s_item = -1;
      bool single = false;
      if (stat) {
        const int first = __shfl_sync(0xffffffffu, edge, 0), last = __shfl_sync(0xffffffffu, edge, 1);
        single = first >= 0 && first == last;
        if (single) {
          s_item = first;
        } else {
          int iv[TC_EROWS / 32];
#pragma unroll
          for (int k = 0; k < TC_EROWS / 32; k++) {
            const int t = t0 + lane + 32 * k;
            iv[k] = t < L_out ? dom_item(a.dout, t) : -1;
          }
#pragma unroll
          for (int k = 0; k < TC_EROWS / 32; k++) eit[lane + 32 * k] = iv[k];
          __syncwarp();
        }
      }
      float s_sum = 0.0f, s_sq = 0.0f;
      auto s_flush = [&]() {
        if (s_item >= 0 && co_ok) {
          atomicAdd(stat + ((long)s_item * a.cout + co) * 2, (double)s_sum);
          atomicAdd(stat + ((long)s_item * a.cout + co) * 2 + 1, (double)s_sq);
        }
        s_item = -1;
        s_sum = 0.0f;
        s_sq = 0.0f;
      };
      auto s_chunk = [&](int r0, const float* vals) {  // statistics of rows r0 .. r0 + TC_EC - 1
        for (int jj = 0; jj < TC_EC; jj++) {
          const int b = eit[r0 + jj];
          if (b != s_item) {
            s_flush();
            s_item = b;
          }
          if (b >= 0) {
            s_sum += vals[jj];
            s_sq = fmaf(vals[jj], vals[jj], s_sq);
          }
        }
      };
      const bool acc_ok = mbar_wait_t(&acc_full[ab], (lt >> 1) & 1, abort_flag, p.err, trc ? &tew : nullptr);
      if (__any_sync(0xffffffffu, !acc_ok)) break;  // warp-uniform: tcgen05.ld below is warp-collective
      tc_fence_after();
      constexpr int ELD = 32;  // accumulator columns per tcgen05.ld
      for (int sc = 0; sc < TC_EROWS / ELD && !bad; sc++) {
        float v[ELD];
        tmem_ld32(tmem + ((uint32_t)(q * 32) << 16) + ab * TC_N + hrow + sc * ELD, v);
        if (sc == TC_EROWS / ELD - 1) {
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(&acc_empty[ab]);  // this warp's half of the accumulator is read
        }
#pragma unroll
        for (int sub = 0; sub < ELD / TC_EC; sub++) {
          const int c = sc * (ELD / TC_EC) + sub;
          const float* rr = rsb;
          long long tq = trc ? clock64() : 0;
          if (need_res) {
            const int sl = rcons % TC_RES_DEPTH;
            const bool got = mbar_wait(&rbar[sl], (rcons / TC_RES_DEPTH) & 1, abort_flag, p.err);
            // warp-uniform, so the warp-collective tcgen05.ld of the next chunk runs on all lanes
            if (__any_sync(0xffffffffu, !got)) bad = true;
            rr = rsb + sl * TC_EC * 32;
          }
          const uint32_t rrl = smem_u32(rr) + 4u * lane;
          if (trc) t_res += clock64() - tq, tq = clock64();
          if (out_mode == OUT_GELU_PRE) {
            // bf16 window planes for the next layer: lane l holds channel co0 + l, which is element
            // 4 * h + l % 4 of chunk l / 4 of 64-channel block co0 / 64 (h = 32-channel half); four
            // lanes make one 8-byte store per row
            const int h = (co0 >> 5) & 1;
            uint8_t* pl = (uint8_t*)a.ypre + ((size_t)((co0 >> 6) * 8 + (lane >> 2)) * a.ypre_rows + PRE_PAD_FRONT) * 16 +
                          h * 8;
#pragma unroll
            for (int jj = 0; jj < TC_EC; jj++) {
              // gelu_new with the hardware tanh (tanh.approx.f32, relative error about 2^-11): the
              // value is rounded to bf16 (2^-9) right after, and the exact tanhf made this epilogue,
              // not the MMA, the FFN projection's limit (its 12 launches 0.5 ms slower per forward)
              const float ga = v[sub * TC_EC + jj] + bias;
              float th;
              asm("tanh.approx.f32 %0, %1;" : "=f"(th) : "f"(0.797884560802865355f * (ga + 0.044715f * ga * ga * ga)));
              const float r = 0.5f * ga * (1.0f + th);
              const float r1 = __shfl_down_sync(0xffffffffu, r, 1);
              const float r2 = __shfl_down_sync(0xffffffffu, r, 2);
              const float r3 = __shfl_down_sync(0xffffffffu, r, 3);
              const int t = t0 + c * TC_EC + jj;
              if ((lane & 3) == 0 && t < L_out && co0 < a.cout) {
                __nv_bfloat162 p0 = __floats2bfloat162_rn(r, r1), p1 = __floats2bfloat162_rn(r2, r3);
                uint2 u;
                memcpy(&u.x, &p0, 4);
                memcpy(&u.y, &p1, 4);
                *reinterpret_cast<uint2*>(pl + (size_t)t * 16) = u;
              }
            }
            continue;
          }
          float* sb = stg + (c & 1) * TC_EC * 32;
          const uint32_t sbl = smem_u32(sb) + (YB ? 2u : 4u) * lane;  // YB: bf16 chunk, 64 bytes a row
          if (lane == 0) bulk_wait_read1();  // the store issued two chunks ago has read sb
          __syncwarp();
          if (trc) t_stbuf += clock64() - tq;
          float vals[TC_EC];
#pragma unroll
          for (int jj = 0; jj < TC_EC; jj++) {
            float r = v[sub * TC_EC + jj] + bias;
            if (out_mode == OUT_ADD && !red) r = lds_f32(rrl + 128u * jj) + r;
            else if (out_mode == OUT_PLUS) r = (r + lds_f32(rrl + 128u * jj)) * oscale;
            else if (out_mode == OUT_GELU) r = gelu_new(r);
            vals[jj] = r;
            if constexpr (YB) {
              const __nv_bfloat16 hb = __float2bfloat16_rn(r);
              unsigned short u;
              memcpy(&u, &hb, 2);
              sts_u16(sbl + 64u * jj, u);
            } else {
              sts_f32(sbl + 128u * jj, r);
            }
          }
          if (stat) {
            if (single) {
#pragma unroll
              for (int jj = 0; jj < TC_EC; jj++) {
                s_sum += vals[jj];
                s_sq = fmaf(vals[jj], vals[jj], s_sq);
              }
            } else {
              s_chunk(c * TC_EC, vals);
            }
          }
          fence_proxy_async();
          __syncwarp();
          if (lane == 0) {
            if (red)
              tma_reduce_add_2d(&p.ymap, co0, t0 + c * TC_EC, sb);
            else
              tma_store_2d(&p.ymap, co0, t0 + c * TC_EC, sb);
            bulk_commit();
          }
          if (need_res) {  // every lane has read this residual slot: refill it
            if (lane == 0 && c + TC_RES_DEPTH < NCH) {
              const int sl = riss % TC_RES_DEPTH;
              mbar_arrive_expect_tx(&rbar[sl], TC_EBOX);
              tma_load_2d(rsb + sl * TC_EC * 32, &p.rmap, co0, t0 + (c + TC_RES_DEPTH) * TC_EC, &rbar[sl]);
            }
            if (c + TC_RES_DEPTH < NCH) riss++;
            rcons++;
          }
        }
      }
      if (stat) s_flush();
    }
    if (lane == 0) {
      for (uint32_t k = rcons; k < riss; k++) {  // residual loads still in flight (abort path)
        const unsigned long long t0 = tc_now();
        while (!mbar_try(&rbar[k % TC_RES_DEPTH], (k / TC_RES_DEPTH) & 1) && tc_now() - t0 < TC_TIMEOUT_NS) {
        }
      }
      bulk_wait_all();  // this warp's stores complete before exit
    }
    if (trc) {
      p.trace[TR_EP_WAIT] = tew;
      p.trace[TR_EP_WORK] = (unsigned long long)(clock64() - t_start) - tew;
      p.trace[TR_EP_RES] = t_res;
      p.trace[TR_EP_STBUF] = t_stbuf;
    }
  } else if (warp >= 4 + TC_NEPI && IM != IN_PRE) {
    // ---------------------------------------------------------------- activation producers
    // Box by box, thread (box row prow = ptid / 8, chunk j = ptid % 8) converts 8 channels of one
    // input row, with the row's item from the tile's row-item table (written by warp 3); with the
    // x2 upsample each input row feeds two window rows. The item's AdaIN coefficients stay in
    // registers until the item changes; they and the Snake alphas come from the shared-memory
    // tables when the layer has them (else from global memory).
    const int ptid = threadIdx.x - (4 + TC_NEPI) * 32;  // 0 .. TC_NPROD * 32 - 1
    const int j = ptid & 7, prow = ptid >> 3;
    const int cin = a.cin, up2 = in_up2, win_rows = p.win_rows;
    const float2* __restrict__ coef = a.coef;
    const float slope = a.slope;
    const bool affine = in_mode == IN_ADAIN_LEAKY || in_mode == IN_ADAIN_SNAKE;
    const bool snake = in_mode == IN_ADAIN_SNAKE;
    const bool leaky_on = in_mode == IN_ADAIN_LEAKY || in_mode == IN_LEAKY_MASK;
    uint32_t xit = 0;
    int in_sl = 0;
    uint32_t in_ph = 0;  // input ring slot and phase parity of the next box
    const bool trc = p.trace && blockIdx.x == 0 && ptid == 0;
    const bool tab = p.tab != 0;
    unsigned long long tpw = 0, tpi = 0;
    const long long t_start = clock64();
    bool ok = true;
    uint32_t lt = 0;
    for (int tile = blockIdx.x; tile < ntiles && ok; tile += gridDim.x, lt++) {
      const InSpan sp = in_span(p, tile, in_up2, BOXR);
      const int bf = lt & 1;
      if (!mbar_wait_t(&meta_full[bf], (lt >> 1) & 1, abort_flag, p.err, trc ? &tpw : nullptr)) break;
      const uint32_t ri = smem_u32(ritem + bf * TC_MAX_WIN);
      const uint32_t ct = smem_u32(ctab + bf * 2 * TC_TAB);
      const int titem = tab ? mitem[bf] : -1;
      for (int cb = 0; cb < p.ncb && ok; cb++, xit++) {
        const int xs = xit % XST;
        if (!mbar_wait_t(&x_empty[xs], ((xit / XST) & 1) ^ 1, abort_flag, p.err, trc ? &tpw : nullptr)) {
          ok = false;
          break;
        }
        const uint32_t xb = smem_u32(xbuf + xs * xbytes) + (uint32_t)j * 16u * (uint32_t)p.win_pad;
        // this thread's 8 channels: chA .. chA + 3 and chA + 32 .. chA + 35
        const int chA = cb * TC_KB + 4 * j;
        int chs[8];
#pragma unroll
        for (int e = 0; e < 8; e++) chs[e] = chA + (e < 4 ? e : 28 + e);
        // channel pairs q = 0 .. 3: (chA, chA + 1), (chA + 2, chA + 3), (chA + 32, chA + 33), (chA + 34, chA + 35)
        float2 al[4], ial[4], ca[4] = {}, cbb[4] = {};
        int cached = -1;
        if (snake) {
          if (tab) {  // (alpha, 1 / alpha) of the four pairs: 4 x 16 bytes
#pragma unroll
            for (int q = 0; q < 4; q++) {
              const float4 q4 = lds_f4(smem_u32(atab) + (uint32_t)((chs[2 * q] >> 1) * 16));
              al[q] = make_float2(q4.x, q4.y), ial[q] = make_float2(q4.z, q4.w);
            }
          } else {
#pragma unroll
            for (int e = 0; e < 8; e++) {
              const float av = chs[e] < cin ? a.alpha[chs[e]] : 1.0f;
              (e & 1 ? al[e >> 1].y : al[e >> 1].x) = av;
              (e & 1 ? ial[e >> 1].y : ial[e >> 1].x) = 1.0f / av;
            }
          }
        }
        // (scale, shift) of this thread's channels for item b: from the tile's table when b is its item
        auto load_coef = [&](int b) {
          if (tab && b == titem) {
#pragma unroll
            for (int q = 0; q < 4; q++) {
              const float4 q4 = lds_f4(ct + (uint32_t)((chs[2 * q] >> 1) * 16));
              ca[q] = make_float2(q4.x, q4.y), cbb[q] = make_float2(q4.z, q4.w);
            }
          } else {
#pragma unroll
            for (int e = 0; e < 8; e++) {
              const float2 q2 = chs[e] < cin ? coef[(long)b * cin + chs[e]] : make_float2(0.0f, 0.0f);
              (e & 1 ? ca[e >> 1].y : ca[e >> 1].x) = q2.x;
              (e & 1 ? cbb[e >> 1].y : cbb[e >> 1].x) = q2.y;
            }
          }
        };
        if (affine && tab && titem >= 0) {
          cached = titem;
          load_coef(titem);
        }
        // prologue of one window row r from the 8 input values v, stored as bf16
        auto emit = [&](int r, const float (&v)[8]) {
          const int b = lds_s32(ri + 4u * (uint32_t)r);
          float o[8];
          if (b < 0) {
#pragma unroll
            for (int e = 0; e < 8; e++) o[e] = 0.0f;
          } else if (affine) {
            if (b != cached) {
              cached = b;
              load_coef(b);
            }
            // packed f32x2 arithmetic (each lane rounds exactly like the scalar fmaf / multiply)
#pragma unroll
            for (int e = 0; e < 8; e += 2) {
              float2 t = __ffma2_rn(make_float2(v[e], v[e + 1]), ca[e >> 1], cbb[e >> 1]);
              if (snake) {
                const float2 arg = __fmul2_rn(al[e >> 1], t);
                const float2 sn = make_float2(__sinf(arg.x), __sinf(arg.y));
                t = __ffma2_rn(ial[e >> 1], __fmul2_rn(sn, sn), t);
              } else {
                t.x = leaky(t.x, slope);
                t.y = leaky(t.y, slope);
              }
              o[e] = t.x;
              o[e + 1] = t.y;
            }
          } else if (leaky_on) {
#pragma unroll
            for (int e = 0; e < 8; e++) o[e] = leaky(v[e], slope);
          } else {
#pragma unroll
            for (int e = 0; e < 8; e++) o[e] = v[e];
          }
          uint4 pk;
          __nv_bfloat162 h0 = __floats2bfloat162_rn(o[0], o[1]);
          __nv_bfloat162 h1 = __floats2bfloat162_rn(o[2], o[3]);
          __nv_bfloat162 h2 = __floats2bfloat162_rn(o[4], o[5]);
          __nv_bfloat162 h3 = __floats2bfloat162_rn(o[6], o[7]);
          memcpy(&pk.x, &h0, 4);
          memcpy(&pk.y, &h1, 4);
          memcpy(&pk.z, &h2, 4);
          memcpy(&pk.w, &h3, 4);
          sts_u4(xb + (uint32_t)r * 16u, pk);
        };
        for (int i = 0; i < sp.nbox; i++) {
          const int sl = in_sl;
          if (!mbar_wait_t(&in_full[sl], in_ph, abort_flag, p.err, trc ? &tpi : nullptr)) {
            ok = false;
            break;
          }
          if (++in_sl == RST) in_sl = 0, in_ph ^= 1;
          const uint32_t box = smem_u32(inring + sl * INBOX) + (uint32_t)(prow * TC_KB + 4 * j) * 4u;
          constexpr int NH = BOXR / TC_PROWS;
          bool done_fast = false;
          if (!up2 && affine) {
            // this thread's rows of the box at once: when every row is a gap or belongs to the
            // cached item, compute all of them unconditionally (interleaved chains) and store with
            // predicates; otherwise fall back to row-by-row emits
            float vv[NH][8];
            int rw[NH], bw[NH];
            bool fast = true;
#pragma unroll
            for (int hh = 0; hh < NH; hh++) {
              const float4 lo = lds_f4(box + (uint32_t)(TC_PROWS * hh * TC_KB) * 4u);
              const float4 hi = lds_f4(box + (uint32_t)(TC_PROWS * hh * TC_KB + 32) * 4u);
              vv[hh][0] = lo.x, vv[hh][1] = lo.y, vv[hh][2] = lo.z, vv[hh][3] = lo.w;
              vv[hh][4] = hi.x, vv[hh][5] = hi.y, vv[hh][6] = hi.z, vv[hh][7] = hi.w;
              rw[hh] = i * BOXR + prow + TC_PROWS * hh;
              bw[hh] = rw[hh] < win_rows ? lds_s32(ri + 4u * (uint32_t)rw[hh]) : -1;
              fast = fast && (bw[hh] < 0 || bw[hh] == cached);
            }
            if (fast) {
              uint4 pk[NH];
#pragma unroll
              for (int hh = 0; hh < NH; hh++) {
                float o[8];
#pragma unroll
                for (int e = 0; e < 8; e += 2) {
                  float2 t = __ffma2_rn(make_float2(vv[hh][e], vv[hh][e + 1]), ca[e >> 1], cbb[e >> 1]);
                  if (snake) {
                    const float2 arg = __fmul2_rn(al[e >> 1], t);
                    const float2 sn = make_float2(__sinf(arg.x), __sinf(arg.y));
                    t = __ffma2_rn(ial[e >> 1], __fmul2_rn(sn, sn), t);
                  } else {
                    t.x = leaky(t.x, slope);
                    t.y = leaky(t.y, slope);
                  }
                  o[e] = t.x;
                  o[e + 1] = t.y;
                }
                __nv_bfloat162 h0 = __floats2bfloat162_rn(o[0], o[1]), h1 = __floats2bfloat162_rn(o[2], o[3]);
                __nv_bfloat162 h2 = __floats2bfloat162_rn(o[4], o[5]), h3 = __floats2bfloat162_rn(o[6], o[7]);
                memcpy(&pk[hh].x, &h0, 4);
                memcpy(&pk[hh].y, &h1, 4);
                memcpy(&pk[hh].z, &h2, 4);
                memcpy(&pk[hh].w, &h3, 4);
                if (bw[hh] < 0) pk[hh] = make_uint4(0u, 0u, 0u, 0u);
              }
#pragma unroll
              for (int hh = 0; hh < NH; hh++)
                if (rw[hh] < win_rows) sts_u4(xb + (uint32_t)rw[hh] * 16u, pk[hh]);
            } else {
#pragma unroll
              for (int hh = 0; hh < NH; hh++)
                if (rw[hh] < win_rows) emit(rw[hh], vv[hh]);
            }
            done_fast = true;
          }
#pragma unroll
          for (int hh = 0; hh < NH && !done_fast; hh++) {
            const int br = prow + TC_PROWS * hh;
            const float4 lo = lds_f4(box + (uint32_t)(TC_PROWS * hh * TC_KB) * 4u);
            const float4 hi = lds_f4(box + (uint32_t)(TC_PROWS * hh * TC_KB + 32) * 4u);
            const float v[8] = {lo.x, lo.y, lo.z, lo.w, hi.x, hi.y, hi.z, hi.w};
            if (!up2) {
              const int r = i * BOXR + br;
              if (r < win_rows) emit(r, v);
            } else {
              const int r0 = 2 * (sp.xr0 + i * BOXR + br) - sp.base;
              if (r0 >= 0 && r0 < win_rows) emit(r0, v);
              if (r0 + 1 >= 0 && r0 + 1 < win_rows) emit(r0 + 1, v);
            }
          }
          __syncwarp();
          if (lane == 0) mbar_arrive(&in_empty[sl]);  // this warp has read the box
        }
        if (!ok) break;
        fence_proxy_async();
        __syncwarp();
        if (lane == 0) mbar_arrive(&x_full[xs]);
      }
      __syncwarp();
      if (ok && lane == 0) mbar_arrive(&meta_empty[bf]);  // this warp is done with the tile's tables
    }
    if (trc) {
      p.trace[TR_PR_WAIT_X] = tpw;
      p.trace[TR_PR_WAIT_IN] = tpi;
      p.trace[TR_PR_WORK] = (unsigned long long)(clock64() - t_start) - tpw - tpi;
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, 512;" ::"r"(tmem) : "memory");
  }
}

// ------------------------------------------------------------------------------ IN_PRE prologue

// Block = 64 plane rows x 128 input channels (two 64-channel blocks), 8 warps. Warp w reads rows
// 8w .. 8w + 7 of the tile as whole 512-byte row segments (lane l: channels 4l .. 4l + 3; all eight
// rows' loads issued before any is used), applies the layer's prologue with the item's
// coefficients cached across rows, and leaves bf16 values in a plane-major shared-memory tile
// (plane stride padded to 65 rows: conflict-free 8-byte stores). Warp w then writes planes 2w and
// 2w + 1: 64 consecutive 16-byte plane rows, 1 KB contiguous each. Reads and writes of HBM
// are both fully coalesced. The kernel issues about as many instructions as the SM can (ncu: issue
// active 75%, DRAM 47% on the 256-channel layers), so per-row work is kept off the lanes: the
// prologue is a template parameter, lane m < 8 looks up the item of row m (a frame-domain lookup
// divides by the domain's scale) and the warp takes it by shuffle, and the AdaIN + Snake arithmetic
// runs on channel pairs in packed f32x2 instructions (each lane rounds like the scalar fmaf /
// multiply, so the planes are bit-identical to the scalar form). Four blocks of 64 rows per SM (64
// registers) keep 256 rows in flight; 32-row blocks held 160-192 and ran the Snake layers 3% slower.
template <int IM>
__global__ void __launch_bounds__(256, 4) prologue_bf16_kernel(const ConvArgs a, uint4* __restrict__ out, long pre_rows,
                                                            int n_planes) {
  __shared__ uint4 tile[16][65];
  constexpr int RW = 8;  // rows per warp
  constexpr bool affine = IM == IN_ADAIN_LEAKY || IM == IN_ADAIN_SNAKE;
  constexpr bool snake = IM == IN_ADAIN_SNAKE;
  constexpr bool leaky_on = IM == IN_ADAIN_LEAKY || IM == IN_LEAKY_MASK;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const long r0 = blockIdx.x * 64L + warp * RW;  // this warp's first plane row
  const int cin = a.cin, c0 = blockIdx.y * 128 + 4 * lane;
  const bool full = c0 + 3 < cin;
  auto row_in = [&](long r) {
    const long g = r - PRE_PAD_FRONT;
    return g >= 0 && g < a.L_in && r < pre_rows;
  };
  int bl = -1;  // lane m < RW: item of row r0 + m
  if (lane < RW && row_in(r0 + lane)) bl = IM == IN_NOMASK ? 0 : dom_item(a.din, (int)(r0 + lane - PRE_PAD_FRONT));
  float4 v[RW];
#pragma unroll
  for (int m = 0; m < RW; m++) {
    const long r = r0 + m, g = r - PRE_PAD_FRONT;
    v[m] = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
    if (row_in(r) && c0 < cin) {
      const long off = (long)(a.in_up2 ? (g >> 1) : g) * a.ldx + c0;
      auto ld4 = [&](const float* base) {
        const float* src = base + off;
        float4 t = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
        if (full) {
          t = __ldg(reinterpret_cast<const float4*>(src));
        } else {
          t.x = __ldg(src);
          if (c0 + 1 < cin) t.y = __ldg(src + 1);
          if (c0 + 2 < cin) t.z = __ldg(src + 2);
        }
        return t;
      };
      v[m] = ld4(a.x);
      if (a.x_b) {  // mean of three resblocks, in the resblock-mean kernel's order of operations
        const float4 vb = ld4(a.x_b), vc = ld4(a.x_c);
        v[m] = make_float4(((v[m].x + vb.x) + vc.x) / 3.0f, ((v[m].y + vb.y) + vc.y) / 3.0f,
                           ((v[m].z + vb.z) + vc.z) / 3.0f, ((v[m].w + vb.w) + vc.w) / 3.0f);
      }
    }
  }
  // channel pairs (c0, c0 + 1) and (c0 + 2, c0 + 3)
  float2 al[2], ial[2];
  if (snake) {
#pragma unroll
    for (int e = 0; e < 4; e++) {
      const float av = c0 + e < cin ? __ldg(a.alpha + c0 + e) : 1.0f;
      (e & 1 ? al[e >> 1].y : al[e >> 1].x) = av;
      (e & 1 ? ial[e >> 1].y : ial[e >> 1].x) = __frcp_rn(av);  // = 1.0f / av (both correctly rounded)
    }
  }
  // plane of lane l's channels within the tile: block l / 16, chunk l % 8, half (l / 8) % 2
  const int tp = (lane >> 4) * 8 + (lane & 7), th = (lane >> 3) & 1;
  float2 qs[2], qh[2];  // AdaIN (scale, shift) of the two channel pairs
  int cached = -1;
#pragma unroll
  for (int m = 0; m < RW; m++) {
    const int b = __shfl_sync(0xffffffffu, bl, m);
    float2 o[2] = {make_float2(v[m].x, v[m].y), make_float2(v[m].z, v[m].w)};
    if (b < 0) {
      o[0] = o[1] = make_float2(0.0f, 0.0f);
    } else if (affine) {
      if (b != cached) {
        cached = b;
#pragma unroll
        for (int e = 0; e < 4; e++) {
          const float2 q = c0 + e < cin ? __ldg(a.coef + (long)b * cin + c0 + e) : make_float2(0.0f, 0.0f);
          (e & 1 ? qs[e >> 1].y : qs[e >> 1].x) = q.x;
          (e & 1 ? qh[e >> 1].y : qh[e >> 1].x) = q.y;
        }
      }
#pragma unroll
      for (int h = 0; h < 2; h++) {
        float2 t = __ffma2_rn(o[h], qs[h], qh[h]);
        if (snake) {
          const float2 arg = __fmul2_rn(al[h], t);
          const float2 sn = make_float2(__sinf(arg.x), __sinf(arg.y));
          t = __ffma2_rn(ial[h], __fmul2_rn(sn, sn), t);
        } else {
          t.x = leaky(t.x, a.slope);
          t.y = leaky(t.y, a.slope);
        }
        o[h] = t;
      }
    } else if (leaky_on) {
#pragma unroll
      for (int h = 0; h < 2; h++) o[h] = make_float2(leaky(o[h].x, a.slope), leaky(o[h].y, a.slope));
    }
    __nv_bfloat162 p0 = __floats2bfloat162_rn(o[0].x, o[0].y), p1 = __floats2bfloat162_rn(o[1].x, o[1].y);
    uint2 u;
    memcpy(&u.x, &p0, 4);
    memcpy(&u.y, &p1, 4);
    reinterpret_cast<uint2*>(&tile[tp][warp * RW + m])[th] = u;
  }
  __syncthreads();
#pragma unroll
  for (int k = 0; k < 4; k++) {
    const int p = 2 * warp + (k >> 1), plane = blockIdx.y * 16 + p, rr = (k & 1) * 32 + lane;
    const long r = blockIdx.x * 64L + rr;
    if (plane < n_planes && r < pre_rows) out[(long)plane * pre_rows + r] = tile[p][rr];
  }
}

cudaError_t launch_prologue_bf16(const ConvArgs& a, void* xpre, long pre_rows, cudaStream_t st) {
  const int ncb = (a.cin + TC_KB - 1) / TC_KB;
  if (a.ldx % 4 != 0 || (((uintptr_t)a.x) & 15) != 0) return cudaErrorInvalidValue;
  const dim3 grid((unsigned)((pre_rows + 63) / 64), (ncb + 1) / 2);
  switch (a.in_mode) {
    case IN_NOMASK: prologue_bf16_kernel<IN_NOMASK><<<grid, 256, 0, st>>>(a, (uint4*)xpre, pre_rows, ncb * 8); break;
    case IN_MASK: prologue_bf16_kernel<IN_MASK><<<grid, 256, 0, st>>>(a, (uint4*)xpre, pre_rows, ncb * 8); break;
    case IN_ADAIN_LEAKY:
      prologue_bf16_kernel<IN_ADAIN_LEAKY><<<grid, 256, 0, st>>>(a, (uint4*)xpre, pre_rows, ncb * 8);
      break;
    case IN_ADAIN_SNAKE:
      prologue_bf16_kernel<IN_ADAIN_SNAKE><<<grid, 256, 0, st>>>(a, (uint4*)xpre, pre_rows, ncb * 8);
      break;
    case IN_LEAKY_MASK:
      prologue_bf16_kernel<IN_LEAKY_MASK><<<grid, 256, 0, st>>>(a, (uint4*)xpre, pre_rows, ncb * 8);
      break;
    default: return cudaErrorInvalidValue;
  }
  return cudaGetLastError();
}

// ------------------------------------------------------------------------------ host side

bool tc_available() {
  int dev = 0, major = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return false;
  if (cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev) != cudaSuccess) return false;
  return major == 10;
}

static inline uint16_t f2bf(float f) {
  uint32_t u;
  memcpy(&u, &f, 4);
  u += 0x7FFFu + ((u >> 16) & 1u);
  return (uint16_t)(u >> 16);
}

// Channel (within its 64-channel block) at K position kp of the operand: chunk kp / 8 holds
// channels 4 * chunk .. + 3 and 32 + 4 * chunk .. + 3 (the producers' conversion order).
static inline int block_channel(int kp) {
  const int j = kp >> 3, e = kp & 7;
  return e < 4 ? 4 * j + e : 32 + 4 * j + (e - 4);
}

cudaError_t tc_make_weights(const float* w, int cin, int cout, int K, TcWeights* out) {
  const int n_cot = (cout + TC_M - 1) / TC_M, ncb = (cin + TC_KB - 1) / TC_KB;
  const size_t n = (size_t)n_cot * ncb * K * (TC_M * TC_KB);
  std::vector<uint16_t> img(n, 0);
  for (int cot = 0; cot < n_cot; cot++)
    for (int cb = 0; cb < ncb; cb++)
      for (int k = 0; k < K; k++) {
        uint16_t* blk = img.data() + (((size_t)cot * ncb + cb) * K + k) * (TC_M * TC_KB);
        for (int r = 0; r < TC_M; r++) {
          const int co = cot * TC_M + r;
          if (co >= cout) continue;
          for (int kp = 0; kp < TC_KB; kp++) {
            const int ci = cb * TC_KB + block_channel(kp);
            if (ci >= cin) continue;
            // chunk kp / 8 at 2048 B, row group r / 8 at 128 B, row r % 8 at 16 B, element kp % 8
            const size_t off = (size_t)(kp >> 3) * 1024 + (size_t)(r >> 3) * 64 + (size_t)(r & 7) * 8 + (kp & 7);
            blk[off] = f2bf(w[((size_t)co * cin + ci) * K + k]);
          }
        }
      }
  void* d = nullptr;
  cudaError_t e = cudaMalloc(&d, n * 2);
  if (e != cudaSuccess) return e;
  e = cudaMemcpy(d, img.data(), n * 2, cudaMemcpyHostToDevice);
  if (e != cudaSuccess) {
    cudaFree(d);
    return e;
  }
  out->w = d;
  out->bytes = n * 2;
  out->cin = cin, out->cout = cout, out->K = K;
  out->cin_pad = ncb * TC_KB, out->cout_pad = n_cot * TC_M;
  return cudaSuccess;
}

typedef void (*TcKernelFn)(const TcArgs);
// Instances for the (input mode, x2 upsample, output mode) combinations the model uses; any other
// combination runs the generic instance.
static TcKernelFn pick_kernel(int im, int up, int om, int* idx) {
  static const struct {
    int im, up, om;
    TcKernelFn fn;
  } table[] = {
      {IN_ADAIN_SNAKE, 0, OUT_STORE, tc_conv_kernel<IN_ADAIN_SNAKE, 0, OUT_STORE>},
      {IN_ADAIN_SNAKE, 0, OUT_ADD, tc_conv_kernel<IN_ADAIN_SNAKE, 0, OUT_ADD>},
      {IN_ADAIN_SNAKE, 0, OUT_PLUS, tc_conv_kernel<IN_ADAIN_SNAKE, 0, OUT_PLUS>},
      {IN_NOMASK, 0, OUT_STORE, tc_conv_kernel<IN_NOMASK, 0, OUT_STORE>},
      {IN_NOMASK, 0, OUT_PLUS, tc_conv_kernel<IN_NOMASK, 0, OUT_PLUS>},
      {IN_NOMASK, 0, OUT_GELU, tc_conv_kernel<IN_NOMASK, 0, OUT_GELU>},
      {IN_ADAIN_LEAKY, 0, OUT_STORE, tc_conv_kernel<IN_ADAIN_LEAKY, 0, OUT_STORE>},
      {IN_ADAIN_LEAKY, 0, OUT_PLUS, tc_conv_kernel<IN_ADAIN_LEAKY, 0, OUT_PLUS>},
      {IN_LEAKY_MASK, 0, OUT_STORE, tc_conv_kernel<IN_LEAKY_MASK, 0, OUT_STORE>},
      {IN_LEAKY_MASK, 0, OUT_PLUS, tc_conv_kernel<IN_LEAKY_MASK, 0, OUT_PLUS>},
      {IN_MASK, 0, OUT_STORE, tc_conv_kernel<IN_MASK, 0, OUT_STORE>},
      {IN_MASK, 1, OUT_STORE, tc_conv_kernel<IN_MASK, 1, OUT_STORE>},
      {IN_PRE, 0, OUT_STORE, tc_conv_kernel<IN_PRE, 0, OUT_STORE>},
      {IN_PRE, 0, OUT_ADD, tc_conv_kernel<IN_PRE, 0, OUT_ADD>},
      {IN_PRE, 0, OUT_PLUS, tc_conv_kernel<IN_PRE, 0, OUT_PLUS>},
      {IN_PRE, 0, OUT_GELU, tc_conv_kernel<IN_PRE, 0, OUT_GELU>},
      {IN_PRE, 0, OUT_GELU_PRE, tc_conv_kernel<IN_PRE, 0, OUT_GELU_PRE>},
      {IN_PRE, 0, OUT_STORE_BF, tc_conv_kernel<IN_PRE, 0, OUT_STORE_BF>},
  };
  const int n = (int)(sizeof(table) / sizeof(table[0]));
  for (int i = 0; i < n; i++)
    if (table[i].im == im && table[i].up == up && table[i].om == om) {
      *idx = i;
      return table[i].fn;
    }
  *idx = n;
  return tc_conv_kernel<-1, 0, -1>;
}

// Input box rows of the instance that runs a layer (the generic instance uses 32).
static int box_rows_of(const ConvArgs& a) {
  const bool pre = a.in_mode == IN_PRE;
  int idx = 0;
  const TcKernelFn fn = pick_kernel(a.in_mode, pre ? 0 : a.in_up2, a.out_mode, &idx);
  return fn == tc_conv_kernel<-1, 0, -1> ? TC_BOX_ROWS : tc_box_rows(a.in_mode, a.out_mode);
}

// Shared memory of one CTA: weight ring, activation windows, input-box ring, epilogue buffers
// (epb bytes per warp), mbarriers (+ TMEM slot, abort flag, table items), the double-buffered
// row-item table and, with tab, the coefficient and alpha tables.
static size_t tc_smem(int win_pad, int rst, int box_rows, int xst, int epb, bool tab) {
  return (size_t)TC_WST * TC_WBLOCK + (size_t)xst * 8 * win_pad * 16 + (size_t)rst * box_rows * TC_KB * 4 +
         (size_t)TC_NEPI * epb + (2 * TC_WST + 2 * TC_RST_MAX + 2 * TC_XST_MAX + 4 + TC_NEPI * TC_RES_DEPTH + 4) * 8 +
         16 + 2 * TC_MAX_WIN * 4 + (tab ? 3 * TC_TAB * 8 : 0);
}

static inline int win_pad_of(int K, int dil) { return ((TC_N + (K - 1) * dil + 7) / 8) * 8 + 1; }

// Input-box ring depth that fits next to the other buffers (0 when even 2 stages do not fit).
static int ring_stages(int win_pad, int box_rows, int epb, bool tab) {
  for (int r = TC_RST_MAX; r >= 2; r--)
    if (tc_smem(win_pad, r, box_rows, 2, epb, tab) <= (size_t)TC_SMEM_MAX) return r;
  return 0;
}

// OUT_ADD layers without fused statistics accumulate by TMA reduce (no residual boxes)
static bool add_by_reduce(const ConvArgs& a) { return a.out_mode == OUT_ADD && !a.stat; }
static int epb_of(const ConvArgs& a) {
  return tc_epi_warp_bytes((a.out_mode == OUT_ADD && !add_by_reduce(a)) || a.out_mode == OUT_PLUS);
}

// The shared-memory coefficient tables serve affine prologues of up to TC_TAB input channels.
static bool tab_of(const ConvArgs& a, int cin_pad) {
  return (a.in_mode == IN_ADAIN_LEAKY || a.in_mode == IN_ADAIN_SNAKE) && cin_pad <= TC_TAB;
}

// Rows of esize-byte elements that TMA can move: 16-byte aligned base and row stride.
static bool rows_ok(const void* base, long ld, int esize = 4) {
  return base && (ld * esize) % 16 == 0 && (((uintptr_t)base) & 15) == 0;
}

bool tc_supported(const ConvArgs& a, const TcWeights& t) {
  if (a.stride != 1 || a.K != t.K || a.cin != t.cin || a.cout != t.cout) return false;
  if (a.L_out < 64) return false;  // tiny row counts (per-item style projections) stay on SIMT
  if ((a.in_mode == IN_ADAIN_LEAKY || a.in_mode == IN_ADAIN_SNAKE) && !a.coef) return false;
  if (TC_N + (a.K - 1) * a.dil > TC_MAX_WIN) return false;
  if (ring_stages(win_pad_of(a.K, a.dil), box_rows_of(a), epb_of(a), tab_of(a, t.cin_pad)) == 0) return false;
  // every global operand moves by TMA: 16-byte aligned bases and row strides
  if (a.in_mode != IN_PRE && !rows_ok(a.x, a.ldx)) return false;
  if (a.out_mode == OUT_GELU_PRE) {
    if (!a.ypre || (((uintptr_t)a.ypre) & 15) != 0 || a.cout % TC_KB != 0 || a.stat) return false;
  } else if (a.out_mode == OUT_STORE_BF) {
    // one instance (IN_PRE input): other inputs take the pre-transform route first (tc_conv refuses
    // them otherwise)
    if (a.stat || a.in_up2 || !rows_ok(a.y, a.ldy, 2)) return false;
  } else if (!rows_ok(a.y, a.ldy)) {
    return false;
  }
  if (a.out_mode == OUT_PLUS && !rows_ok(a.sc, a.ldsc)) return false;
  return true;
}

static int g_num_sms[64] = {0};
static unsigned g_attr_set[64] = {0};  // per device: instances whose shared-memory limit is raised

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static bool tried = false;
  if (!tried) {
    tried = true;
    void* f = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &f, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = (EncodeTiledFn)f;
    else
      cudaGetLastError();
  }
  return fn;
}

// f32 rows [rows][cols] with row stride ld floats; box = box_cols x box_rows, no swizzle; elements
// outside the tensor read as zero.
static bool make_rows_map(CUtensorMap* m, const void* base, long rows, long cols, long ld, int box_cols,
                          int box_rows, bool bf16_rows = false) {
  EncodeTiledFn fn = encode_fn();
  const int es = bf16_rows ? 2 : 4;
  if (!fn || !rows_ok(base, ld, es) || rows <= 0 || cols <= 0) return false;
  cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)ld * es};
  cuuint32_t box[2] = {(cuuint32_t)box_cols, (cuuint32_t)box_rows};
  cuuint32_t estr[2] = {1, 1};
  return fn(m, bf16_rows ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, (void*)base, dims,
            strides, box, estr,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_128B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

cudaError_t tc_conv(const ConvArgs& a, const TcWeights& t, int* err, cudaStream_t st, unsigned long long* trace) {
  if (!tc_supported(a, t)) return cudaErrorInvalidValue;
  TcArgs p;
  memset(&p, 0, sizeof(p));
  p.trace = trace;
  const long x_rows = a.in_up2 ? (a.L_in + 1) / 2 : a.L_in;
  const bool pre = a.in_mode == IN_PRE;
  if (pre && (!a.xpre || (((uintptr_t)a.xpre) & 15) != 0)) return cudaErrorInvalidValue;
  if (a.out_mode == OUT_STORE_BF && !pre) return cudaErrorInvalidValue;  // its one instance reads IN_PRE planes
  if (a.x_b && !pre) return cudaErrorInvalidValue;  // the three-input mean is formed by the pre-transform
  const int box_rows = box_rows_of(a);
  bool maps = (pre || make_rows_map(&p.xmap, a.x, x_rows, a.cin, a.ldx, TC_KB, box_rows)) &&
              (a.out_mode == OUT_GELU_PRE ||
               make_rows_map(&p.ymap, a.y, a.L_out, a.cout, a.ldy, 32, TC_EC, a.out_mode == OUT_STORE_BF));
  if (maps && a.out_mode == OUT_ADD) maps = make_rows_map(&p.rmap, a.y, a.L_out, a.cout, a.ldy, 32, TC_EC);
  if (maps && a.out_mode == OUT_PLUS) maps = make_rows_map(&p.rmap, a.sc, a.L_out, a.cout, a.ldsc, 32, TC_EC);
  if (!maps) return cudaErrorInvalidValue;
  p.a = a;
  p.wimg = (const __nv_bfloat16*)t.w;
  p.ncb = t.cin_pad / TC_KB;
  p.n_cot = t.cout_pad / TC_M;
  p.n_tt = (a.L_out + TC_N - 1) / TC_N;
  p.win_rows = TC_N + (a.K - 1) * a.dil;
  p.win_pad = win_pad_of(a.K, a.dil);
  p.err = err;
  p.epb = epb_of(a);
  p.red = add_by_reduce(a) ? 1 : 0;
  p.tab = !pre && tab_of(a, t.cin_pad);
  p.rst = pre ? 0 : ring_stages(p.win_pad, box_rows, p.epb, p.tab);
  p.xst = 2;
  if (pre)  // no input ring: spend its shared memory on deeper window staging
    while (p.xst < TC_XST_MAX && tc_smem(p.win_pad, 0, box_rows, p.xst + 1, p.epb, false) <= (size_t)TC_SMEM_MAX)
      p.xst++;
  const size_t smem = tc_smem(p.win_pad, p.rst, box_rows, p.xst, p.epb, p.tab);
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 64 && g_num_sms[dev] == 0) {
    int n = 0;
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    g_num_sms[dev] = n;
  }
  int ci = 0;
  const TcKernelFn fn = pick_kernel(a.in_mode, pre ? 0 : a.in_up2, a.out_mode, &ci);
  if (dev < 64 && !(g_attr_set[dev] & (1u << ci))) {
    cudaError_t e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, TC_SMEM_MAX);
    if (e != cudaSuccess) return e;
    g_attr_set[dev] |= 1u << ci;
  }
  const int ntiles = p.n_cot * p.n_tt;
  const int nsm = g_num_sms[dev < 64 ? dev : 0];
  const int grid = ntiles < nsm ? ntiles : nsm;
  fn<<<grid, TC_THREADS, smem, st>>>(p);
  return cudaGetLastError();
}

}  // namespace kk
