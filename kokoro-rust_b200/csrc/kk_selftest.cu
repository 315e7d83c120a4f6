// Diagnostics entry point: one 1-D convolution through the tcgen05 kernel on caller buffers, so the
// kernel can be checked on its own against an fp32 reference (every prologue / epilogue mode, odd
// channel counts, ragged item layouts). Not part of the model path.
#include <cuda_runtime.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>
#include <string>
#include <algorithm>
#include <vector>

#include "../../include/kokoro_b200.h"
#include "kk_common.cuh"
#include "kk_launch.h"
#include "kk_tc.h"

#include "kk_tc_ptx.cuh"

namespace kk {

// One thread initialises an mbarrier that expects one arrival, then waits on its first phase with
// the bounded wait every tcgen05 pipeline uses; nothing ever arrives, so the wait must give up after
// limit_ns, raise the error flag and return (no trap, no fault, no TMA or TMEM in flight).
__global__ void wait_selftest_kernel(int* err, unsigned long long limit_ns) {
  __shared__ __align__(8) uint64_t bar;
  __shared__ int abort_flag;
  if (threadIdx.x == 0) {
    mbar_init(&bar, 1);
    abort_flag = 0;
  }
  __syncthreads();
  if (threadIdx.x == 0) mbar_wait_lim(&bar, 0, &abort_flag, err, limit_ns);
  __syncthreads();
}

cudaError_t launch_wait_selftest(int* err, unsigned long long limit_ns, cudaStream_t st) {
  wait_selftest_kernel<<<1, 32, 0, st>>>(err, limit_ns);
  return cudaGetLastError();
}

}  // namespace kk

namespace {

thread_local std::string g_selftest_error;

struct DevBuf {
  void* p = nullptr;
  ~DevBuf() {
    if (p) cudaFree(p);
  }
};

kk_status fail(kk_status s, const std::string& m) {
  g_selftest_error = m;
  return s;
}

}  // namespace

extern "C" KK_API const char* kk_conv_selftest_error(void) { return g_selftest_error.c_str(); }

extern "C" KK_API kk_status kk_conv_selftest(int cuda_ordinal, const kk_conv_case* c, const float* x,
                                             const float* w, const float* bias, const float* coef,
                                             const float* alpha, const float* sc, float* y, double* stat,
                                             int timing_iters, double* ms_per_iter) {
  using namespace kk;
  if (!c || !x || !w || !y) return fail(KK_ERR_INVALID_ARG, "null argument");
  if (c->cin < 1 || c->cout < 1 || c->K < 1 || c->dil < 1 || c->rows_in < 1 || c->rows_out < 1 ||
      c->ldx < c->cin || c->ldy < c->cout || c->n_items < 1 || !c->item_in || !c->item_out)
    return fail(KK_ERR_INVALID_ARG, "bad shape");
  const bool affine = c->in_mode == IN_ADAIN_LEAKY || c->in_mode == IN_ADAIN_SNAKE;
  if (affine && !coef) return fail(KK_ERR_INVALID_ARG, "AdaIN modes need coef");
  if (c->in_mode == IN_ADAIN_SNAKE && !alpha) return fail(KK_ERR_INVALID_ARG, "Snake needs alpha");
  if (c->out_mode == OUT_PLUS && (!sc || c->ldsc < c->cout)) return fail(KK_ERR_INVALID_ARG, "PLUS needs sc");
  if (cudaSetDevice(cuda_ordinal) != cudaSuccess || !tc_available())
    return fail(KK_ERR_CUDA, "no compute-capability-10 device");
  cudaStream_t st = nullptr;
  const long xrows = c->up2 ? (c->rows_in + 1) / 2 : c->rows_in;
  DevBuf dx, dw, db, dcoef, dal, dsc, dy, dst, dii, dio, derr;
  auto put = [&](DevBuf& b, const void* h, size_t n) -> bool {
    if (cudaMalloc(&b.p, n) != cudaSuccess) return false;
    return cudaMemcpy(b.p, h, n, cudaMemcpyHostToDevice) == cudaSuccess;
  };
  bool ok = put(dx, x, sizeof(float) * xrows * c->ldx) && put(dy, y, sizeof(float) * (size_t)c->rows_out * c->ldy) &&
            put(dii, c->item_in, sizeof(int) * c->rows_in) && put(dio, c->item_out, sizeof(int) * c->rows_out);
  if (ok && bias) ok = put(db, bias, sizeof(float) * c->cout);
  if (ok && affine) ok = put(dcoef, coef, sizeof(float) * 2 * (size_t)c->n_items * c->cin);
  if (ok && alpha) ok = put(dal, alpha, sizeof(float) * c->cin);
  if (ok && c->out_mode == OUT_PLUS) ok = put(dsc, sc, sizeof(float) * (size_t)c->rows_out * c->ldsc);
  if (ok && stat) ok = cudaMalloc(&dst.p, sizeof(double) * 2 * (size_t)c->n_items * c->cout) == cudaSuccess &&
                       cudaMemset(dst.p, 0, sizeof(double) * 2 * (size_t)c->n_items * c->cout) == cudaSuccess;
  if (ok) ok = cudaMalloc(&derr.p, sizeof(int)) == cudaSuccess && cudaMemset(derr.p, 0, sizeof(int)) == cudaSuccess;
  if (!ok) return fail(KK_ERR_OOM, "device allocation / copy failed");

  TcWeights t;
  cudaError_t e = tc_make_weights(w, c->cin, c->cout, c->K, &t);
  if (e != cudaSuccess) return fail(KK_ERR_CUDA, cudaGetErrorString(e));
  DevBuf dimg;
  dimg.p = t.w;

  ConvArgs a;
  memset(&a, 0, sizeof(a));
  a.x = (const float*)dx.p, a.ldx = c->ldx, a.cin = c->cin, a.L_in = c->rows_in;
  a.in_mode = c->in_mode, a.in_up2 = c->up2, a.slope = c->slope;
  a.coef = (const float2*)dcoef.p, a.alpha = (const float*)dal.p;
  a.din = Dom{(const int*)dii.p, 0, 0, 0, c->rows_in};
  a.w = nullptr, a.bias = (const float*)db.p, a.cout = c->cout, a.K = c->K, a.dil = c->dil, a.pad = c->pad,
  a.stride = 1;
  a.y = (float*)dy.p, a.ldy = c->ldy, a.L_out = c->rows_out, a.out_mode = c->out_mode;
  a.sc = (const float*)dsc.p, a.ldsc = c->ldsc, a.oscale = c->oscale;
  a.stat = (double*)dst.p;
  a.dout = Dom{(const int*)dio.p, 0, 0, 0, c->rows_out};
  if (!tc_supported(a, t)) return fail(KK_ERR_INVALID_ARG, "shape not supported by the tcgen05 kernel");
  DevBuf dpre;
  if (c->pre) {
    a.pre_rows = PRE_PAD_FRONT + (long)c->rows_in + PRE_PAD_BACK;
    if (cudaMalloc(&dpre.p, (size_t)((c->cin + 63) / 64) * 8 * a.pre_rows * 16) != cudaSuccess)
      return fail(KK_ERR_OOM, "device allocation failed");
    e = launch_prologue_bf16(a, dpre.p, a.pre_rows, st);
    if (e != cudaSuccess) return fail(KK_ERR_CUDA, cudaGetErrorString(e));
    a.xpre = dpre.p;
    a.in_mode = IN_PRE;
    a.in_up2 = 0;
  }
  // KK_TC_TRACE=1 (diagnostics): per-role cycle accounting of CTA 0, printed to stderr
  DevBuf dtr;
  if (getenv("KK_TC_TRACE") && cudaMalloc(&dtr.p, 16 * sizeof(unsigned long long)) == cudaSuccess)
    cudaMemset(dtr.p, 0, 16 * sizeof(unsigned long long));
  e = tc_conv(a, t, (int*)derr.p, st, (unsigned long long*)dtr.p);
  if (e == cudaSuccess) e = cudaStreamSynchronize(st);
  if (e != cudaSuccess) return fail(KK_ERR_CUDA, cudaGetErrorString(e));
  if (dtr.p) {
    unsigned long long h[16];
    if (cudaMemcpy(h, dtr.p, sizeof(h), cudaMemcpyDeviceToHost) == cudaSuccess) {
      fprintf(stderr, "tc_trace K=%d dil=%d cin=%d cout=%d L=%d in=%d out=%d |", a.K, a.dil, a.cin, a.cout, a.L_out,
              a.in_mode, a.out_mode);
      for (int i = 0; i < 16; i++) fprintf(stderr, " %llu", h[i]);
      fprintf(stderr, "\n");
    }
  }
  if (timing_iters > 0 && ms_per_iter) {
    // repeated launches on the same buffers (out_mode 1 keeps accumulating; the first result is
    // the one returned below only when timing_iters == 0)
    cudaEvent_t e0, e1;
    cudaEventCreate(&e0);
    cudaEventCreate(&e1);
    cudaEventRecord(e0, st);
    for (int i = 0; i < timing_iters && e == cudaSuccess; i++) {
      if (c->pre) {  // the input transform is part of every launch of the pre route
        ConvArgs a0 = a;
        a0.in_mode = c->in_mode, a0.in_up2 = c->up2;
        e = launch_prologue_bf16(a0, dpre.p, a.pre_rows, st);
        if (e != cudaSuccess) break;
      }
      e = tc_conv(a, t, (int*)derr.p, st);
    }
    cudaEventRecord(e1, st);
    if (e == cudaSuccess) e = cudaEventSynchronize(e1);
    float ms = 0;
    cudaEventElapsedTime(&ms, e0, e1);
    cudaEventDestroy(e0);
    cudaEventDestroy(e1);
    if (e != cudaSuccess) return fail(KK_ERR_CUDA, cudaGetErrorString(e));
    *ms_per_iter = ms / timing_iters;
  }
  int errh = 0;
  if (cudaMemcpy(&errh, derr.p, sizeof(int), cudaMemcpyDeviceToHost) != cudaSuccess)
    return fail(KK_ERR_CUDA, "error flag read failed");
  if (errh) return fail(KK_ERR_TIMEOUT, "a tcgen05 pipeline wait timed out");
  if (cudaMemcpy(y, dy.p, sizeof(float) * (size_t)c->rows_out * c->ldy, cudaMemcpyDeviceToHost) != cudaSuccess)
    return fail(KK_ERR_CUDA, "output copy failed");
  if (stat && cudaMemcpy(stat, dst.p, sizeof(double) * 2 * (size_t)c->n_items * c->cout, cudaMemcpyDeviceToHost) !=
                  cudaSuccess)
    return fail(KK_ERR_CUDA, "statistics copy failed");
  return KK_OK;
}

// qkv_bf16: qkv holds bf16 bit patterns (2 bytes per element) instead of f32.
static kk_status attention_selftest(int cuda_ordinal, int n_items, const int32_t* tok_len, const void* qkv,
                                    bool qkv_bf16, float* ctx) {
  using namespace kk;
  if (n_items < 1 || !tok_len || !qkv || !ctx) return fail(KK_ERR_INVALID_ARG, "null argument");
  std::vector<ItemTab> items(n_items);
  std::vector<int2> wl[3];
  int rows = 0;
  for (int b = 0; b < n_items; b++) {
    const int T = tok_len[b];
    if (T < 1 || T > 512) return fail(KK_ERR_INVALID_ARG, "item length outside [1, 512]");
    items[b] = ItemTab{rows, T, 0, 0};
    const int k = T <= 128 ? 0 : (T <= 256 ? 1 : 2);
    for (int q0 = 0; q0 < T; q0 += 128) wl[k].push_back(make_int2(b, q0));
    rows += T;
  }
  std::vector<int2> all;
  int n_work[3];
  for (int k = 0; k < 3; k++) {
    n_work[k] = (int)wl[k].size();
    all.insert(all.end(), wl[k].begin(), wl[k].end());
  }
  if (cudaSetDevice(cuda_ordinal) != cudaSuccess || !tc_available())
    return fail(KK_ERR_CUDA, "no compute-capability-10 device");
  DevBuf dq, dc, di, dw, derr;
  auto put = [&](DevBuf& b, const void* h, size_t n) -> bool {
    if (cudaMalloc(&b.p, n) != cudaSuccess) return false;
    return cudaMemcpy(b.p, h, n, cudaMemcpyHostToDevice) == cudaSuccess;
  };
  bool ok = put(dq, qkv, (qkv_bf16 ? 2 : 4) * (size_t)rows * 2304) && put(di, items.data(), sizeof(ItemTab) * n_items) &&
            put(dw, all.data(), sizeof(int2) * all.size()) &&
            cudaMalloc(&dc.p, sizeof(float) * rows * 768) == cudaSuccess &&
            cudaMemset(dc.p, 0, sizeof(float) * rows * 768) == cudaSuccess &&
            cudaMalloc(&derr.p, sizeof(int)) == cudaSuccess && cudaMemset(derr.p, 0, sizeof(int)) == cudaSuccess;
  if (!ok) return fail(KK_ERR_OOM, "device allocation / copy failed");
  cudaError_t e = launch_attention_tc(dq.p, 2304, qkv_bf16, (const ItemTab*)di.p, (const int2*)dw.p, n_work,
                                      (float*)dc.p, 768, (int*)derr.p, nullptr);
  if (e == cudaSuccess) e = cudaDeviceSynchronize();
  if (e != cudaSuccess) return fail(KK_ERR_CUDA, cudaGetErrorString(e));
  int errh = 0;
  cudaMemcpy(&errh, derr.p, sizeof(int), cudaMemcpyDeviceToHost);
  if (errh) return fail(KK_ERR_TIMEOUT, "a tcgen05 attention wait timed out");
  if (cudaMemcpy(ctx, dc.p, sizeof(float) * rows * 768, cudaMemcpyDeviceToHost) != cudaSuccess)
    return fail(KK_ERR_CUDA, "output copy failed");
  return KK_OK;
}

extern "C" KK_API kk_status kk_attention_selftest(int cuda_ordinal, int n_items, const int32_t* tok_len,
                                                  const float* qkv, float* ctx) {
  return attention_selftest(cuda_ordinal, n_items, tok_len, qkv, false, ctx);
}

extern "C" KK_API kk_status kk_attention_selftest_bf16(int cuda_ordinal, int n_items, const int32_t* tok_len,
                                                       const uint16_t* qkv, float* ctx) {
  return attention_selftest(cuda_ordinal, n_items, tok_len, qkv, true, ctx);
}

extern "C" KK_API kk_status kk_lstm_selftest(int cuda_ordinal, int tc, int n_items, const int32_t* len,
                                             const float* gx, const float* whh, const float* bhh, float* out) {
  using namespace kk;
  if (n_items < 1 || n_items > LSTM_IPG || !len || !gx || !whh || !bhh || !out)
    return fail(KK_ERR_INVALID_ARG, "bad arguments (1 to 32 items)");
  if (tc)
    for (size_t i = 0; i < (size_t)2 * 1024 * 256; i++)
      if (!(fabsf(whh[i]) <= 32768.0f)) return fail(KK_ERR_INVALID_ARG, "tc = 1 needs |whh| <= 2^15 (fp16 split operands)");
  int rows = 0, Tmax = 0;
  std::vector<int> gstart(LSTM_IPG, 0), glen(LSTM_IPG, 0);
  std::vector<int> order(n_items);
  for (int b = 0; b < n_items; b++) {
    if (len[b] < 1) return fail(KK_ERR_INVALID_ARG, "item length < 1");
    order[b] = b;
  }
  std::vector<int> start(n_items);
  for (int b = 0; b < n_items; b++) start[b] = rows, rows += len[b], Tmax = len[b] > Tmax ? len[b] : Tmax;
  // longest first within the group, as the engine orders it
  for (int i = 0; i < n_items; i++)
    for (int j = i + 1; j < n_items; j++)
      if (len[order[j]] > len[order[i]]) std::swap(order[i], order[j]);
  for (int r = 0; r < n_items; r++) gstart[r] = start[order[r]], glen[r] = len[order[r]];
  std::vector<int> gact(Tmax);
  for (int s2 = 0; s2 < Tmax; s2++) {
    int n = 0;
    while (n < LSTM_IPG && glen[n] > s2) n++;
    gact[s2] = n;
  }
  if (cudaSetDevice(cuda_ordinal) != cudaSuccess || (tc && !tc_available()))
    return fail(KK_ERR_CUDA, "no suitable device");
  DevBuf dgx, dw, db, dout, dgs, dgl, dga, derr;
  auto put = [&](DevBuf& b, const void* h, size_t n) -> bool {
    if (cudaMalloc(&b.p, n) != cudaSuccess) return false;
    return cudaMemcpy(b.p, h, n, cudaMemcpyHostToDevice) == cudaSuccess;
  };
  bool ok = put(dgx, gx, sizeof(float) * rows * 2048) && put(dw, whh, sizeof(float) * 2 * 1024 * 256) &&
            put(db, bhh, sizeof(float) * 2 * 1024) && put(dgs, gstart.data(), sizeof(int) * LSTM_IPG) &&
            put(dgl, glen.data(), sizeof(int) * LSTM_IPG) && put(dga, gact.data(), sizeof(int) * Tmax) &&
            cudaMalloc(&dout.p, sizeof(float) * rows * 512) == cudaSuccess &&
            cudaMemset(dout.p, 0, sizeof(float) * rows * 512) == cudaSuccess &&
            cudaMalloc(&derr.p, sizeof(int)) == cudaSuccess && cudaMemset(derr.p, 0, sizeof(int)) == cudaSuccess;
  if (!ok) return fail(KK_ERR_OOM, "device allocation / copy failed");
  LstmArgs a;
  memset(&a, 0, sizeof(a));
  a.gx = (const float*)dgx.p, a.ldgx = 2048, a.whh = (const float*)dw.p, a.bhh = (const float*)db.p;
  a.out = (float*)dout.p, a.ldo = 512, a.gstart = (const int*)dgs.p, a.glen = (const int*)dgl.p;
  a.gact = (const int*)dga.p, a.G = 1, a.IPG = LSTM_IPG, a.Tmax = Tmax, a.tc = tc, a.err = (int*)derr.p;
  cudaError_t e = launch_lstm(a, nullptr);
  if (e == cudaSuccess) e = cudaDeviceSynchronize();
  if (e != cudaSuccess) return fail(KK_ERR_CUDA, cudaGetErrorString(e));
  int errh = 0;
  cudaMemcpy(&errh, derr.p, sizeof(int), cudaMemcpyDeviceToHost);
  if (errh) return fail(KK_ERR_TIMEOUT, "an LSTM MMA wait timed out");
  if (cudaMemcpy(out, dout.p, sizeof(float) * rows * 512, cudaMemcpyDeviceToHost) != cudaSuccess)
    return fail(KK_ERR_CUDA, "output copy failed");
  return KK_OK;
}
