// kokoro-b200 engine: weight hydration, per-engine device arena, and the batched ragged forward
// behind the C ABI of include/kokoro_b200.h.
//
// The forward follows GpuKokoro::forward_batch (src/gpu_batch.rs:179-421) stage by stage, with
// one B200-first change of representation: every activation is time-major ([rows][channels]),
// so a convolution tap is a row offset, a linear layer is a 1-tap convolution, a channel concat
// is a column range of one buffer, and the transposes of the reference disappear.
#include <cmath>
#include <cstdio>
#include <cstring>
#include <algorithm>
#include <memory>
#include <mutex>
#include <numeric>
#include <thread>
#include <string>
#include <vector>

#include "../../include/kokoro_b200.h"
#include "kk_common.cuh"
#include "kk_launch.h"
#include "kk_tc.h"
#include "kk_weights.h"

namespace kk {

// Copies n[i] bytes from src[i] to dst[i] for every i on up to 8 host threads, split into
// contiguous runs of items of about equal bytes: the destinations are usually freshly allocated
// caller arrays, so the page faults of first touch dominate and are served in parallel.
static void parallel_copy(int count, void* const* dst, const void* const* src, const size_t* n) {
  size_t total = 0;
  for (int i = 0; i < count; i++) total += n[i];
  const size_t per_thread = size_t(8) << 20;  // below 8 MiB a thread is not worth starting
  // up to 16 threads (the first touch of fresh destination pages dominates, and it scales with
  // threads); KK_FETCH_THREADS caps it, e.g. to the cores per process when several engines share
  // one host
  static const size_t cap = [] {
    const char* e = getenv("KK_FETCH_THREADS");
    const long v = e ? strtol(e, nullptr, 10) : 16;
    return (size_t)std::max(1L, std::min(64L, v));
  }();
  int T = (int)std::min<size_t>({cap, (size_t)std::max(1u, std::thread::hardware_concurrency()),
                                 std::max<size_t>(1, total / per_thread)});
  if (T <= 1 || count <= 1) {
    for (int i = 0; i < count; i++) memcpy(dst[i], src[i], n[i]);
    return;
  }
  std::vector<std::thread> th;
  int first = 0;
  size_t done = 0;
  for (int t = 0; t < T && first < count; t++) {
    const size_t goal = total * (size_t)(t + 1) / (size_t)T;
    int last = first;
    size_t acc = done;
    while (last < count && (acc < goal || last == first)) acc += n[last++];
    if (t == T - 1) last = count;
    th.emplace_back([=] {
      for (int i = first; i < last; i++) memcpy(dst[i], src[i], n[i]);
    });
    for (int i = first; i < last; i++) done += n[i];
    first = last;
  }
  for (auto& x : th) x.join();
}

#define KK_CUDA(expr)                                                                         \
  do {                                                                                        \
    cudaError_t _e = (expr);                                                                  \
    if (_e != cudaSuccess) {                                                                  \
      throw ::kk::KKError(_e == cudaErrorMemoryAllocation ? KK_ERR_OOM : KK_ERR_CUDA,               \
                    std::string(#expr) + ": " + cudaGetErrorString(_e));                      \
    }                                                                                         \
  } while (0)

#define KK_REQUIRE(cond, msg)                                   \
  do {                                                          \
    if (!(cond)) throw ::kk::KKError(KK_ERR_INVALID_ARG, (msg));      \
  } while (0)

// ------------------------------------------------------------------------------ device arena

// Bump allocator over a chain of cudaMalloc'd blocks, kept across calls; mark/rewind give
// stack-like reuse inside a forward (safe because all work is ordered on one stream).
class Arena {
 public:
  ~Arena() { release(); }
  void release() {
    for (auto& b : blocks_) cudaFree(b.p);
    blocks_.clear();
    cur_ = 0;
  }
  // External-block mode: allocations are carved from one caller-provided device block and never
  // reach cudaMalloc; exhausting the block throws. Only kk_decode_batch_noalloc uses it.
  void set_external(void* base, size_t cap) {
    ext_base_ = static_cast<char*>(base);
    ext_cap_ = cap;
    ext_used_ = 0;
  }
  void clear_external() { ext_base_ = nullptr; }
  // Gap canary (tests): with a stream set, every buffer handed out is first filled with NaN bytes on
  // that stream, so an element read before any kernel wrote it poisons the result.
  void set_poison(cudaStream_t st) { poison_st_ = st; }
  void* alloc(size_t bytes) {
    void* p = alloc_raw(bytes);
    if (poison_st_) {
      cudaError_t e = cudaMemsetAsync(p, 0xFF, (bytes + 255) & ~size_t(255), poison_st_);
      if (e != cudaSuccess) throw KKError(KK_ERR_CUDA, std::string("gap canary fill: ") + cudaGetErrorString(e));
    }
    return p;
  }
  void* alloc_raw(size_t bytes) {
    bytes = (bytes + 255) & ~size_t(255);
    if (bytes == 0) bytes = 256;
    if (ext_base_) {
      // the peak statistic describes the allocating arena only, never the static scratch
      if (ext_used_ + bytes > ext_cap_)
        throw KKError(KK_ERR_INVALID_ARG, "static scratch exhausted (batch above the no-allocation limit)");
      void* p = ext_base_ + ext_used_;
      ext_used_ += bytes;
      return p;
    }
    while (cur_ < blocks_.size()) {
      Block& b = blocks_[cur_];
      if (b.used + bytes <= b.cap) {
        void* p = b.p + b.used;
        b.used += bytes;
        note_peak();
        return p;
      }
      cur_++;
    }
    size_t last = blocks_.empty() ? 0 : blocks_.back().cap;
    size_t cap = std::max({bytes, 2 * last, size_t(256) << 20});
    char* p = nullptr;
    cudaError_t e = cudaMalloc(&p, cap);
    if (e != cudaSuccess) {
      cudaGetLastError();
      cap = bytes;
      e = cudaMalloc(&p, cap);
      if (e != cudaSuccess) {
        cudaGetLastError();
        throw KKError(KK_ERR_OOM, "device arena: cannot allocate " + std::to_string(bytes >> 20) + " MiB");
      }
    }
    blocks_.push_back({p, cap, bytes});
    cur_ = blocks_.size() - 1;
    note_peak();
    return p;
  }
  template <class T>
  T* get(size_t n) {
    return static_cast<T*>(alloc(n * sizeof(T)));
  }
  struct Mark {
    size_t blk, used;
  };
  Mark mark() const {
    if (ext_base_) return {~size_t(0), ext_used_};
    return {cur_, cur_ < blocks_.size() ? blocks_[cur_].used : 0};
  }
  void rewind(Mark m) {
    if (ext_base_) {
      ext_used_ = m.used;
      return;
    }
    for (size_t i = m.blk + 1; i < blocks_.size(); i++) blocks_[i].used = 0;
    if (m.blk < blocks_.size()) blocks_[m.blk].used = m.used;
    cur_ = m.blk;
  }
  void reset() {
    for (auto& b : blocks_) b.used = 0;
    cur_ = 0;
    peak_ = 0;
  }
  size_t bytes() const {
    size_t s = 0;
    for (auto& b : blocks_) s += b.cap;
    return s;
  }
  // Largest number of bytes in use at once since the last reset (the device memory a call needs
  // beyond the weights; the free-VRAM batch budget is derived from it).
  size_t peak() const { return peak_; }

 private:
  void note_peak() {
    size_t u = 0;
    for (size_t i = 0; i <= cur_ && i < blocks_.size(); i++) u += blocks_[i].used;
    if (u > peak_) peak_ = u;
  }
  struct Block {
    char* p;
    size_t cap, used;
  };
  std::vector<Block> blocks_;
  size_t cur_ = 0;
  char* ext_base_ = nullptr;
  size_t ext_cap_ = 0, ext_used_ = 0;
  size_t peak_ = 0;
  cudaStream_t poison_st_ = nullptr;
};

// Pinned host staging for the uploads and downloads of one call (reset per call).
class PinnedArena {
 public:
  ~PinnedArena() {
    for (auto& b : blocks_) cudaFreeHost(b.p);
  }
  void* alloc(size_t bytes) {
    bytes = (bytes + 63) & ~size_t(63);
    for (; cur_ < blocks_.size(); cur_++) {
      if (blocks_[cur_].used + bytes <= blocks_[cur_].cap) {
        void* p = blocks_[cur_].p + blocks_[cur_].used;
        blocks_[cur_].used += bytes;
        return p;
      }
    }
    size_t cap = std::max(bytes, size_t(64) << 20);
    char* p = nullptr;
    if (cudaHostAlloc(&p, cap, cudaHostAllocDefault) != cudaSuccess) {
      cudaGetLastError();
      throw KKError(KK_ERR_OOM, "pinned host staging: cannot allocate " + std::to_string(cap >> 20) + " MiB");
    }
    blocks_.push_back({p, cap, bytes});
    cur_ = blocks_.size() - 1;
    return p;
  }
  void reset() {
    for (auto& b : blocks_) b.used = 0;
    cur_ = 0;
  }

 private:
  struct Block {
    char* p;
    size_t cap, used;
  };
  std::vector<Block> blocks_;
  size_t cur_ = 0;
};

// ------------------------------------------------------------------------------ model

struct Conv {
  int cin = 0, cout = 0, K = 1, dil = 1, pad = 0, stride = 1;
  bool simt_only = false;  // always the fp32 kernel (the per-item style projections: one row per item)
  double macs_per_row = 0;  // algorithmic multiply-adds per output row
  float* w = nullptr;  // fp32 [K][cin][cout]
  float* b = nullptr;
  TcWeights tc;        // bf16 tcgen05 operand layout (BF16 precision only)
};
struct AdaIN {
  float* nw = nullptr;
  float* nb = nullptr;
  int off = 0;  // column offset of this layer's gamma|beta in the fused per-item fc output
  int c = 0;
};
struct ResBlk {
  int din = 0, dout = 0;
  bool up = false, has_sc = false;
  Conv c1, c2, sc;
  AdaIN n1, n2;
  float* pool_w = nullptr;
  float* pool_b = nullptr;
};
struct SnakeBlk {
  int c = 0, k = 0;
  Conv c1[3], c2[3];
  AdaIN a1[3], a2[3];
  float* al1[3];
  float* al2[3];
};
struct Lstm {
  Conv ih;  // both directions: cout = 2 * 4H (W_ih fwd | W_ih reverse), bias b_ih
  float* whh = nullptr;
  float* bhh = nullptr;
  bool f16_ok = false;  // every |W_hh| <= 2^15: the tensor-core recurrence's fp16 split operands hold it
};

struct Model {
  float *word, *pos, *tt0, *emb_g, *emb_b;
  Conv map_in, qkv, dense, ffn, ffn_out;
  float *attn_g, *attn_b, *full_g, *full_b;
  Conv bert_enc;
  Lstm dur_lstm[3];
  int adaln_off[3];
  Lstm pred_lstm, shared, te_lstm;
  Conv dur_proj;
  ResBlk f0[3], nn[3];
  Conv f0_proj, n_proj;
  float* te_emb;
  Conv te_cnn[3];
  float *te_g[3], *te_b[3];
  ResBlk enc, dec[4];
  float *f0conv_w, *nconv_w;
  float f0conv_b, nconv_b;
  Conv asr_res;
  float* lw;
  float lb;
  Conv noise0, noise1, ups[2], post;
  Conv noise0_rows;  // BF16 mode: noise_convs.0 as a 2-tap conv over 6-frame rows (see load)
  SnakeBlk noise_res[2], rb[6];
  Conv fc_dec, fc_pro;  // all AdaIN / AdaLN style projections fused: cin 128, cout = sum of 2C
};

static const int DILS[3] = {1, 3, 5};
// Row strides of the decoder's channel-concatenation buffers, rounded up to 16 bytes so that
// tensor-memory-access copies and vector loads apply: [asr | f0 | n] (514 channels) and
// [x | asr_res | f0 | n] (1090 channels).
static const int X0_LD = 516;
static const int CAT_LD = 1092;
// Row strides of the spectrum (22 channels) and of conv_post's output (22 channels), padded to
// 16 bytes so the tensor-core convolutions can move them with TMA.
static const int SPEC_LD = 24;
static const int POST_LD = 24;
static inline int ld16(int c) { return (c + 3) & ~3; }  // row stride of a c-channel f32 buffer
// Layers with more output channels than this pre-transform their input once (IN_PRE) instead of
// in the conv's producer warps (which redo it for every 128-channel output tile); so do the K <= 3
// layers of exactly this many. Measured on B200 (kk_conv_selftest, 300,000 rows): at 256 channels
// with K = 3 the pre-transform route is 10% faster (its MMAs are too few to hide two transforms per
// input element), with K = 7 / 11 the fused route is 9-13% faster; from 512 channels on the
// pre-transform route is 1.7x faster.
static const int TC_PRE_MIN_COUT = 256;
// The token and frame layouts hold at least this many rows (trailing gap rows make up the rest):
// the tensor-core path takes layers of 64 rows or more, so in BF16 mode every layer runs the same
// arithmetic whatever the size of the batch (a one-item batch of a short line would otherwise run
// its token-domain layers on the fp32 kernel and give a different result than the same line in a
// larger batch).
static const int MIN_LAYOUT_ROWS = 64;

struct Engine {
  int dev = 0;
  int precision = KK_PRECISION_FP32;
  cudaStream_t st = nullptr;
  Model m{};
  std::vector<void*> wallocs;
  size_t wbytes = 0;
  Arena ar;
  PinnedArena pin;
  std::string err;
  std::string ident;
  bool keep_audio_dev = false, sync_each = false;
  bool pcm16_out = false;                // KK_OPT_OUTPUT_PCM16
  bool gap_canary = false;               // KK_OPT_GAP_CANARY (tests): arena buffers start as NaN
  bool negctl_nomask = false;            // KK_OPT_NEGCTL_NOMASK (tests, FP32 mode): convs read gap rows unmasked
  bool attn_f32 = false;                 // KK_OPT_ATTENTION_F32 (diagnostics): BF16 mode with the fp32 attention
  int16_t* audio_host16 = nullptr;       // pinned PCM_16 of the last forward
  size_t audio_host16_cap = 0;
  std::vector<long long> out_clipped;    // per item, with KK_OPT_OUTPUT_PCM16
  long long launches = 0;
  int* err_flag = nullptr;
  bool tc_ok = false;
  bool noalloc_active = false;  // inside kk_decode_batch_noalloc: no events, no pinned staging
  const char* tc_trace_dir = getenv("KK_TC_TRACE_DIR");  // diagnostics: per-launch pipeline cycle accounting
  const bool prof_shapes = getenv("KK_PROFILE_SHAPES") != nullptr;  // diagnostics: conv shape in the class name
  int cur_B = 0;  // items of the batch being run
  long long last_tokens = 0, last_frames = 0;  // sizes of the last call (memory statistics)
  // timing: events on the engine stream (begin, compute begin, compute end, end)
  cudaEvent_t ev[4] = {nullptr, nullptr, nullptr, nullptr};
  double last_times[4] = {0, 0, 0, 0};
  double h2d_bytes = 0, d2h_bytes = 0;
  bool profile = false;
  struct ProfRec {
    int cls;
    cudaEvent_t a, b;
    double flops, bytes;
  };
  struct ProfLaunch {  // one timed launch since the last profile reset
    int cls;
    double ms, flops, bytes;
  };
  std::vector<ProfLaunch> prof_log;
  std::vector<ProfRec> prof_pending;
  std::vector<cudaEvent_t> ev_pool;
  size_t ev_used = 0;
  std::vector<std::string> prof_names;
  std::vector<long long> prof_launches;
  std::vector<double> prof_ms, prof_flops;
  cudaEvent_t stage_ev = nullptr;  // profile: the last stage boundary (intervals become "stage:<name>")
  // results of the last forward
  float* audio_host = nullptr;
  size_t audio_host_cap = 0;
  std::vector<long long> out_off, out_len;

  ~Engine();
  // -- load
  float* up(const std::vector<float>& v);
  Conv conv_from(const std::vector<float>& w, const float* bias_h, int cin, int cout, int K, int dil, int pad,
                 int stride);
  Conv load_conv(const Checkpoint& ck, const std::string& p, int cin, int cout, int K, int dil, int pad, int stride,
                 bool bias);
  Conv load_linear(const Checkpoint& ck, const std::string& p, int din, int dout, bool bias = true);
  AdaIN load_adain(const Checkpoint& ck, const std::string& p, int c, std::vector<float>& fcw, std::vector<float>& fcb);
  ResBlk load_resblk(const Checkpoint& ck, const std::string& p, int din, int dout, bool up, std::vector<float>& fcw,
                     std::vector<float>& fcb);
  SnakeBlk load_snake(const Checkpoint& ck, const std::string& p, int c, int k, std::vector<float>& fcw,
                      std::vector<float>& fcb);
  Lstm load_lstm(const Checkpoint& ck, const std::string& p, int din);
  void load(const Checkpoint& ck);
  // -- forward helpers
  template <class T>
  T* upload(const T* h, size_t n);
  void check(cudaError_t e, const char* what);
  void dump(const char* name, const void* p, long long rows, int cols, int ld);
  cudaEvent_t pool_event();
  int prof_class(const char* name);
  void prof_begin(cudaEvent_t* a);
  void prof_end(cudaEvent_t a, const char* cls, double flops, double bytes = 0.0);
  void prof_collect();
  void times_begin();
  void times_compute_begin();
  void times_compute_end();
  void stage_sync(const char* what);
  ConvArgs ca(const Conv& c);
  void run_conv(const Conv& c, ConvArgs& a);
  bool tc_route(const Conv& c, const ConvArgs& a) const;
  bool tc_pre(const Conv& c, const ConvArgs& a) const;
  void run_conv_stats(const Conv& c, ConvArgs& a, const Dom& dout, const ItemTab* items, int B, int max_len,
                      float** mean, float** rstd);
  void stats(const float* x, int ldx, int C, const Dom& d, const ItemTab* items, int B, int max_len, float** mean,
             float** rstd);
  void adain_args(ConvArgs& a, const AdaIN& n, const float* mean, const float* rstd, const float* gb, int ldgb, int mode,
                  float slope, const float* alpha);
  void resblk(const ResBlk& R, const float* x, int ldx, const Dom& din, const Dom& dout, float* y, int ldy,
              const float* gb, int ldgb, const ItemTab* items, int B, int max_n);
  // in_mean / in_rstd: statistics of xin when the caller already has them (shared by parallel blocks)
  void snake(const SnakeBlk& S, const float* xin, float* out, const Dom& d, const float* gb, int ldgb,
             const ItemTab* items, int B, int max_n, const float* in_mean = nullptr, const float* in_rstd = nullptr);
  void lstm(const Lstm& L, const float* x, int ldx, int rows, const std::vector<int>& start,
            const std::vector<int>& len, float* out, int ldo);
  void linear(const Conv& c, const float* x, int ldx, int rows, float* y, int ldy, int out_mode = OUT_STORE,
              const float* sc = nullptr, int ldsc = 0);
  float* decode_core(int B, const std::vector<ItemTab>& items_h, const ItemTab* items, const int* col_item_n, int LN,
                     float* xcat0, float* f0, float* nc, const float* gb_dec, int ldgb, const uint64_t* seeds_d,
                     const float* noise_d, const long long* noise_off_d);
  float* decode_core(int B, int max_n, const ItemTab* items, const int* col_item_n, int LN, float* xcat0, float* f0,
                     float* nc, const float* gb_dec, int ldgb, const uint64_t* seeds_d, const float* noise_d,
                     const long long* noise_off_d);
  // pcm16: honour KK_OPT_OUTPUT_PCM16 (the forward); the vocoder entry returns f32 to its caller
  void finish_audio(float* audio_d, int LN, const std::vector<ItemTab>& items_h, const int* col_item_n, bool pcm16);
  // noise: null, or per item a pointer to replayed draws (null = the item's counter stream) with
  // noise_len[b] floats, checked against 600 * 9 * N_b once the durations are known
  void forward(int B, const int64_t* ids, const int32_t* ids_len, const float* ref_s, const float* speed,
               const uint64_t* seeds, const float* const* noise, const int64_t* noise_len, const float* rand_ini,
               const int64_t* forced, int64_t* dur_out, int64_t* nsamp_out);
  void decode(int B, const int32_t* n_frames, const float* asr, const float* f0, const float* n, const float* s_dec,
              const uint64_t* seeds, const float* noise, float* audio_out);
  void decode_noalloc(int B, const int32_t* n_frames, const float* asr, const float* f0, const float* n,
                      const float* s_dec, const uint64_t* seeds, const float* noise, float* audio_out);
  void wait_selftest(long long limit_ns);
  // replayed noise of the items that carry it (noise[b] != null), -1 offsets for counter-noise items
  void upload_noise(int B, const std::vector<ItemTab>& items_h, const float* const* noise, float** noise_d,
                    long long** noise_off_d);
};

// Message of a nonzero engine error flag (set by a bounded in-kernel wait that gave up).
static std::string wait_error(int code) {
  switch (code) {
    case 2: return "a tcgen05 pipeline barrier wait timed out (error flag 2)";
    case 3: return "a tensor-core attention MMA wait timed out (error flag 3)";
    case 4: return "an LSTM recurrence wait timed out (error flag 4)";
    default: return "a bounded device wait timed out (error flag " + std::to_string(code) + ")";
  }
}

Engine::~Engine() {
  if (dev >= 0) cudaSetDevice(dev);
  if (st) cudaStreamSynchronize(st);
  for (void* p : wallocs) cudaFree(p);
  ar.release();
  if (audio_host) cudaFreeHost(audio_host);
  if (audio_host16) cudaFreeHost(audio_host16);
  for (auto e : ev)
    if (e) cudaEventDestroy(e);
  for (auto e : ev_pool) cudaEventDestroy(e);
  if (st) cudaStreamDestroy(st);
}

cudaEvent_t Engine::pool_event() {
  if (ev_used == ev_pool.size()) {
    cudaEvent_t e;
    KK_CUDA(cudaEventCreate(&e));
    ev_pool.push_back(e);
  }
  return ev_pool[ev_used++];
}

int Engine::prof_class(const char* name) {
  for (size_t i = 0; i < prof_names.size(); i++)
    if (prof_names[i] == name) return (int)i;
  prof_names.push_back(name);
  prof_launches.push_back(0);
  prof_ms.push_back(0);
  prof_flops.push_back(0);
  return (int)prof_names.size() - 1;
}

void Engine::prof_begin(cudaEvent_t* a) {
  *a = nullptr;
  if (!profile || noalloc_active) return;
  *a = pool_event();
  KK_CUDA(cudaEventRecord(*a, st));
}

void Engine::prof_end(cudaEvent_t a, const char* cls, double flops, double bytes) {
  if (!profile || !a) return;
  cudaEvent_t b = pool_event();
  KK_CUDA(cudaEventRecord(b, st));
  prof_pending.push_back({prof_class(cls), a, b, flops, bytes});
}

// Called after the stream is synchronised: fold the recorded launch intervals into the profile.
void Engine::prof_collect() {
  for (auto& r : prof_pending) {
    float ms = 0;
    KK_CUDA(cudaEventElapsedTime(&ms, r.a, r.b));
    prof_launches[r.cls]++;
    prof_ms[r.cls] += ms;
    prof_flops[r.cls] += r.flops;
    prof_log.push_back({r.cls, (double)ms, r.flops, r.bytes});
  }
  prof_pending.clear();
  ev_used = 0;
}

void Engine::times_begin() {
  h2d_bytes = d2h_bytes = 0;
  for (auto& e : ev)
    if (!e) KK_CUDA(cudaEventCreate(&e));
  KK_CUDA(cudaEventRecord(ev[0], st));
}
void Engine::times_compute_begin() {
  if (noalloc_active) return;
  KK_CUDA(cudaEventRecord(ev[1], st));
  stage_ev = nullptr;
  if (profile) {
    stage_ev = pool_event();
    KK_CUDA(cudaEventRecord(stage_ev, st));
  }
}
void Engine::times_compute_end() {
  if (noalloc_active) return;
  KK_CUDA(cudaEventRecord(ev[2], st));
}

float* Engine::up(const std::vector<float>& v) {
  float* p = nullptr;
  KK_CUDA(cudaMalloc(&p, std::max<size_t>(v.size(), 1) * sizeof(float)));
  wallocs.push_back(p);
  wbytes += v.size() * sizeof(float);
  KK_CUDA(cudaMemcpy(p, v.data(), v.size() * sizeof(float), cudaMemcpyHostToDevice));
  return p;
}

// w: torch layout [cout][cin][K] -> fp32 [K][cin][cout] (+ the bf16 tcgen05 layout in BF16 mode)
Conv Engine::conv_from(const std::vector<float>& w, const float* bias_h, int cin, int cout, int K, int dil, int pad,
                       int stride) {
  Conv c;
  c.cin = cin, c.cout = cout, c.K = K, c.dil = dil, c.pad = pad, c.stride = stride;
  c.macs_per_row = (double)cin * cout * K;
  std::vector<float> t((size_t)K * cin * cout);
  for (int co = 0; co < cout; co++)
    for (int ci = 0; ci < cin; ci++)
      for (int k = 0; k < K; k++) t[((size_t)k * cin + ci) * cout + co] = w[((size_t)co * cin + ci) * K + k];
  c.w = up(t);
  if (bias_h) c.b = up(std::vector<float>(bias_h, bias_h + cout));
  if (precision == KK_PRECISION_BF16 && tc_ok) {
    KK_CUDA(tc_make_weights(w.data(), cin, cout, K, &c.tc));
    wallocs.push_back(c.tc.w);
    wbytes += c.tc.bytes;
  }
  return c;
}

Conv Engine::load_conv(const Checkpoint& ck, const std::string& p, int cin, int cout, int K, int dil, int pad,
                       int stride, bool bias) {
  std::vector<float> w = ck.conv_weight(p, {cout, cin, K});
  std::vector<float> b;
  if (bias) b = ck.get(p + ".bias", {cout});
  return conv_from(w, bias ? b.data() : nullptr, cin, cout, K, dil, pad, stride);
}

Conv Engine::load_linear(const Checkpoint& ck, const std::string& p, int din, int dout, bool bias) {
  std::vector<float> w = ck.get(p + ".weight", {dout, din});
  std::vector<float> b;
  if (bias) b = ck.get(p + ".bias", {dout});
  return conv_from(w, bias ? b.data() : nullptr, din, dout, 1, 1, 0, 1);
}

// AdaIN1d (src/nn.rs:87-100): affine defaults, and fc rows appended to the fused projection.
AdaIN Engine::load_adain(const Checkpoint& ck, const std::string& p, int c, std::vector<float>& fcw,
                         std::vector<float>& fcb) {
  AdaIN a;
  a.c = c;
  a.nw = up(ck.norm_affine(p + ".norm.weight", c, 1.0f));
  a.nb = up(ck.norm_affine(p + ".norm.bias", c, 0.0f));
  std::vector<float> w = ck.get(p + ".fc.weight", {2 * c, STYLE});
  std::vector<float> b = ck.get(p + ".fc.bias", {2 * c});
  a.off = (int)fcb.size();
  fcw.insert(fcw.end(), w.begin(), w.end());
  fcb.insert(fcb.end(), b.begin(), b.end());
  return a;
}

// AdainResBlk1d (src/nn.rs:103-141)
ResBlk Engine::load_resblk(const Checkpoint& ck, const std::string& p, int din, int dout, bool upb,
                           std::vector<float>& fcw, std::vector<float>& fcb) {
  ResBlk r;
  r.din = din, r.dout = dout, r.up = upb;
  r.c1 = load_conv(ck, p + ".conv1", din, dout, 3, 1, 1, 1, true);
  r.c2 = load_conv(ck, p + ".conv2", dout, dout, 3, 1, 1, 1, true);
  r.n1 = load_adain(ck, p + ".norm1", din, fcw, fcb);
  r.n2 = load_adain(ck, p + ".norm2", dout, fcw, fcb);
  r.has_sc = din != dout;
  if (r.has_sc) r.sc = load_conv(ck, p + ".conv1x1", din, dout, 1, 1, 0, 1, false);
  if (upb) {
    r.pool_w = up(ck.conv_weight(p + ".pool", {din, 1, 3}));
    r.pool_b = up(ck.get(p + ".pool.bias", {din}));
  }
  if (r.up && !r.has_sc) throw KKError(KK_ERR_IO, p + ": upsampling block without a 1x1 shortcut");
  return r;
}

// AdaINResBlock1 (src/nn.rs:143-166)
SnakeBlk Engine::load_snake(const Checkpoint& ck, const std::string& p, int c, int k, std::vector<float>& fcw,
                            std::vector<float>& fcb) {
  SnakeBlk s;
  s.c = c, s.k = k;
  for (int i = 0; i < 3; i++) {
    int d = DILS[i];
    s.c1[i] = load_conv(ck, p + ".convs1." + std::to_string(i), c, c, k, d, (k * d - d) / 2, 1, true);
    s.c2[i] = load_conv(ck, p + ".convs2." + std::to_string(i), c, c, k, 1, (k - 1) / 2, 1, true);
  }
  for (int i = 0; i < 3; i++) s.a1[i] = load_adain(ck, p + ".adain1." + std::to_string(i), c, fcw, fcb);
  for (int i = 0; i < 3; i++) s.a2[i] = load_adain(ck, p + ".adain2." + std::to_string(i), c, fcw, fcb);
  for (int i = 0; i < 3; i++) s.al1[i] = up(ck.get(p + ".alpha1." + std::to_string(i), {1, c, 1}));
  for (int i = 0; i < 3; i++) s.al2[i] = up(ck.get(p + ".alpha2." + std::to_string(i), {1, c, 1}));
  return s;
}

// BiLSTM (src/nn.rs:170-189): W_ih of both directions stacked into one 1-tap conv (cout 2048).
Lstm Engine::load_lstm(const Checkpoint& ck, const std::string& p, int din) {
  const int H = 256;
  Lstm l;
  std::vector<float> wih, bih, whh, bhh;
  for (const char* sfx : {"", "_reverse"}) {
    auto a = ck.get(p + ".weight_ih_l0" + sfx, {4 * H, din});
    auto b = ck.get(p + ".bias_ih_l0" + sfx, {4 * H});
    auto c = ck.get(p + ".weight_hh_l0" + sfx, {4 * H, H});
    auto d = ck.get(p + ".bias_hh_l0" + sfx, {4 * H});
    wih.insert(wih.end(), a.begin(), a.end());
    bih.insert(bih.end(), b.begin(), b.end());
    whh.insert(whh.end(), c.begin(), c.end());
    bhh.insert(bhh.end(), d.begin(), d.end());
  }
  l.ih = conv_from(wih, bih.data(), din, 8 * H, 1, 1, 0, 1);
  l.whh = up(whh);
  l.bhh = up(bhh);
  float wmax = 0.0f;
  for (float v : whh) wmax = std::max(wmax, std::fabs(v));
  l.f16_ok = wmax <= 32768.0f;  // NaN fails the test too
  return l;
}

// ConvTranspose1d(cin, cout, K, stride s, pad p) as a polyphase 3-tap convolution over the input
// rows (pad 1): output row s*q + j, channel co, is column j*cout + co of input row q, with
// W'[m][ci][j*cout + co] = W_T[ci][co][s*(1 - m) + j + p] when that tap index lies in [0, K).
static void convT_polyphase(const std::vector<float>& wT, const std::vector<float>& b, int cin, int cout, int K, int s,
                            int p, std::vector<float>& w_out, std::vector<float>& b_out) {
  const int cp = s * cout;
  w_out.assign((size_t)cp * cin * 3, 0.0f);  // torch layout [cp][cin][3]
  for (int m = 0; m < 3; m++)
    for (int j = 0; j < s; j++) {
      int k = s * (1 - m) + j + p;
      if (k < 0 || k >= K) continue;
      for (int ci = 0; ci < cin; ci++)
        for (int co = 0; co < cout; co++)
          w_out[((size_t)(j * cout + co) * cin + ci) * 3 + m] = wT[((size_t)ci * cout + co) * K + k];
    }
  b_out.resize(cp);
  for (int j = 0; j < s; j++)
    for (int co = 0; co < cout; co++) b_out[j * cout + co] = b[co];
}

void Engine::load(const Checkpoint& ck) {
  const std::string L = "bert.encoder.albert_layer_groups.0.albert_layers.0";
  std::vector<float> fdw, fdb, fpw, fpb;  // fused style projections: decoder (s_dec), prosody (s_pro)
  // ---- ALBERT (src/albert.rs:36-64)
  m.word = up(ck.get("bert.embeddings.word_embeddings.weight", {178, 128}));
  m.pos = up(ck.get("bert.embeddings.position_embeddings.weight", {512, 128}));
  {
    auto tt = ck.get("bert.embeddings.token_type_embeddings.weight", {2, 128});
    tt.resize(128);
    m.tt0 = up(tt);
  }
  m.emb_g = up(ck.get("bert.embeddings.LayerNorm.weight", {128}));
  m.emb_b = up(ck.get("bert.embeddings.LayerNorm.bias", {128}));
  m.map_in = load_linear(ck, "bert.encoder.embedding_hidden_mapping_in", 128, 768);
  {
    std::vector<float> w, b;
    for (const char* n : {"query", "key", "value"}) {
      auto a = ck.get(L + ".attention." + n + ".weight", {768, 768});
      auto c = ck.get(L + ".attention." + n + ".bias", {768});
      w.insert(w.end(), a.begin(), a.end());
      b.insert(b.end(), c.begin(), c.end());
    }
    m.qkv = conv_from(w, b.data(), 768, 2304, 1, 1, 0, 1);
  }
  m.dense = load_linear(ck, L + ".attention.dense", 768, 768);
  m.attn_g = up(ck.get(L + ".attention.LayerNorm.weight", {768}));
  m.attn_b = up(ck.get(L + ".attention.LayerNorm.bias", {768}));
  m.ffn = load_linear(ck, L + ".ffn", 768, 2048);
  m.ffn_out = load_linear(ck, L + ".ffn_output", 2048, 768);
  m.full_g = up(ck.get(L + ".full_layer_layer_norm.weight", {768}));
  m.full_b = up(ck.get(L + ".full_layer_layer_norm.bias", {768}));
  m.bert_enc = load_linear(ck, "bert_encoder", 768, 512);
  // ---- predictor (src/model.rs:60-86)
  for (int i = 0; i < 3; i++) {
    m.dur_lstm[i] = load_lstm(ck, "predictor.text_encoder.lstms." + std::to_string(2 * i), 640);
    auto w = ck.get("predictor.text_encoder.lstms." + std::to_string(2 * i + 1) + ".fc.weight", {1024, 128});
    auto b = ck.get("predictor.text_encoder.lstms." + std::to_string(2 * i + 1) + ".fc.bias", {1024});
    m.adaln_off[i] = (int)fpb.size();
    fpw.insert(fpw.end(), w.begin(), w.end());
    fpb.insert(fpb.end(), b.begin(), b.end());
  }
  m.pred_lstm = load_lstm(ck, "predictor.lstm", 640);
  m.dur_proj = load_linear(ck, "predictor.duration_proj.linear_layer", 512, 50);
  m.shared = load_lstm(ck, "predictor.shared", 640);
  const char* names[2] = {"F0", "N"};
  for (int s = 0; s < 2; s++) {
    ResBlk* blk = s == 0 ? m.f0 : m.nn;
    std::string p = std::string("predictor.") + names[s];
    blk[0] = load_resblk(ck, p + ".0", 512, 512, false, fpw, fpb);
    blk[1] = load_resblk(ck, p + ".1", 512, 256, true, fpw, fpb);
    blk[2] = load_resblk(ck, p + ".2", 256, 256, false, fpw, fpb);
  }
  m.f0_proj = load_conv(ck, "predictor.F0_proj", 256, 1, 1, 1, 0, 1, true);
  m.n_proj = load_conv(ck, "predictor.N_proj", 256, 1, 1, 1, 0, 1, true);
  // ---- text encoder (src/model.rs:29-44)
  m.te_emb = up(ck.get("text_encoder.embedding.weight", {178, 512}));
  for (int i = 0; i < 3; i++) {
    std::string p = "text_encoder.cnn." + std::to_string(i);
    m.te_cnn[i] = load_conv(ck, p + ".0", 512, 512, 5, 1, 2, 1, true);
    m.te_g[i] = up(ck.get(p + ".1.gamma", {512}));
    m.te_b[i] = up(ck.get(p + ".1.beta", {512}));
  }
  m.te_lstm = load_lstm(ck, "text_encoder.lstm", 512);
  // ---- decoder (src/vocoder.rs:98-111)
  m.enc = load_resblk(ck, "decoder.encode", 514, 1024, false, fdw, fdb);
  for (int i = 0; i < 4; i++)
    m.dec[i] = load_resblk(ck, "decoder.decode." + std::to_string(i), 1090, i < 3 ? 1024 : 512, i == 3, fdw, fdb);
  {
    auto w = ck.conv_weight("decoder.F0_conv", {1, 1, 3});
    m.f0conv_w = up(w);
    m.f0conv_b = ck.get("decoder.F0_conv.bias", {1})[0];
    auto w2 = ck.conv_weight("decoder.N_conv", {1, 1, 3});
    m.nconv_w = up(w2);
    m.nconv_b = ck.get("decoder.N_conv.bias", {1})[0];
  }
  m.asr_res = load_conv(ck, "decoder.asr_res.0", 512, 64, 1, 1, 0, 1, true);
  // ---- generator (src/vocoder.rs:54-80)
  const std::string g = "decoder.generator";
  m.lw = up(ck.get(g + ".m_source.l_linear.weight", {1, 9}));
  m.lb = ck.get(g + ".m_source.l_linear.bias", {1})[0];
  m.noise0 = load_conv(ck, g + ".noise_convs.0", 22, 256, 12, 1, 3, 6, true);
  if (precision == KK_PRECISION_BF16 && tc_ok) {
    // Conv1d(22 -> 256, k12, stride 6, pad 3) over the spectrum rows equals a 2-tap stride-1 conv
    // over "6-frame rows" X'[q] = spec rows 6q-3 .. 6q+2 (6 * SPEC_LD channels: frame j, channel c
    // at j * SPEC_LD + c; the 2 padding channels of each frame are zero in the spectrum and get zero
    // weights): y[o] = W'_0 X'[o] + W'_1 X'[o+1] with W'_m[co][j * SPEC_LD + c] = W[co][c][6m + j].
    // With 3 zero rows ahead of the spectrum, X' is a plain strided view (row stride 6 * SPEC_LD).
    auto w = ck.conv_weight(g + ".noise_convs.0", {256, 22, 12});
    auto b = ck.get(g + ".noise_convs.0.bias", {256});
    const int cv = 6 * SPEC_LD;
    std::vector<float> w2((size_t)256 * cv * 2, 0.0f);
    for (int co = 0; co < 256; co++)
      for (int mm = 0; mm < 2; mm++)
        for (int j = 0; j < 6; j++)
          for (int c = 0; c < 22; c++)
            w2[((size_t)co * cv + j * SPEC_LD + c) * 2 + mm] = w[((size_t)co * 22 + c) * 12 + 6 * mm + j];
    m.noise0_rows = conv_from(w2, b.data(), cv, 256, 2, 1, 0, 1);
    m.noise0_rows.macs_per_row = (double)22 * 256 * 12;
  }
  m.noise1 = load_conv(ck, g + ".noise_convs.1", 22, 128, 1, 1, 0, 1, true);
  m.noise_res[0] = load_snake(ck, g + ".noise_res.0", 256, 7, fdw, fdb);
  m.noise_res[1] = load_snake(ck, g + ".noise_res.1", 128, 11, fdw, fdb);
  const int ups_cfg[2][5] = {{512, 256, 20, 10, 5}, {256, 128, 12, 6, 3}};
  for (int i = 0; i < 2; i++) {
    const int ci = ups_cfg[i][0], co = ups_cfg[i][1], K = ups_cfg[i][2], s = ups_cfg[i][3], p = ups_cfg[i][4];
    std::string pre = g + ".ups." + std::to_string(i);
    auto wT = ck.conv_weight(pre, {ci, co, K});
    auto b = ck.get(pre + ".bias", {co});
    std::vector<float> wp, bp;
    convT_polyphase(wT, b, ci, co, K, s, p, wp, bp);
    m.ups[i] = conv_from(wp, bp.data(), ci, s * co, 3, 1, 1, 1);
    m.ups[i].macs_per_row = (double)ci * co * K;  // ConvTranspose taps per input row
  }
  const int ks[3] = {3, 7, 11};
  for (int i = 0; i < 2; i++)
    for (int j = 0; j < 3; j++)
      m.rb[i * 3 + j] = load_snake(ck, g + ".resblocks." + std::to_string(i * 3 + j), 512 >> (i + 1), ks[j], fdw, fdb);
  m.post = load_conv(ck, g + ".conv_post", 128, 22, 7, 1, 3, 1, true);
  // fused style projections: one row per item, so in fp32 on the SIMT kernel whatever the batch
  // size (the tensor-core path would take them only for batches of 64 items or more)
  m.fc_dec = conv_from(fdw, fdb.data(), 128, (int)fdb.size(), 1, 1, 0, 1);
  m.fc_pro = conv_from(fpw, fpb.data(), 128, (int)fpb.size(), 1, 1, 0, 1);
  m.fc_dec.simt_only = m.fc_pro.simt_only = true;
  KK_CUDA(upload_stft_constants(st));
  KK_CUDA(cudaStreamSynchronize(st));
}

// ------------------------------------------------------------------------------ forward helpers

template <class T>
T* Engine::upload(const T* h, size_t n) {
  T* d = ar.get<T>(std::max<size_t>(n, 1));
  if (n == 0) return d;
  void* s = pin.alloc(n * sizeof(T));
  memcpy(s, h, n * sizeof(T));
  KK_CUDA(cudaMemcpyAsync(d, s, n * sizeof(T), cudaMemcpyHostToDevice, st));
  h2d_bytes += (double)(n * sizeof(T));
  return d;
}

void Engine::check(cudaError_t e, const char* what) {
  launches++;
  if (e != cudaSuccess) throw KKError(e == cudaErrorMemoryAllocation ? KK_ERR_OOM : KK_ERR_CUDA,
                                      std::string(what) + ": " + cudaGetErrorString(e));
  if (sync_each) {
    cudaError_t s = cudaStreamSynchronize(st);
    if (s != cudaSuccess) throw KKError(KK_ERR_CUDA, std::string(what) + " (sync): " + cudaGetErrorString(s));
  }
}

// Diagnostic stage dump: with KK_DEBUG_DUMP_DIR set, copy a [rows][ld] f32 buffer to the host
// and write <dir>/<name>.f32 plus <name>.shape ("rows cols ld").
void Engine::dump(const char* name, const void* p, long long rows, int cols, int ld) {
  const char* dir = getenv("KK_DEBUG_DUMP_DIR");
  if (!dir || !*dir) return;
  KK_CUDA(cudaStreamSynchronize(st));
  std::vector<float> h((size_t)rows * ld);
  KK_CUDA(cudaMemcpy(h.data(), p, h.size() * sizeof(float), cudaMemcpyDeviceToHost));
  std::string base = std::string(dir) + "/" + name;
  FILE* f = fopen((base + ".f32").c_str(), "wb");
  if (f) {
    fwrite(h.data(), sizeof(float), h.size(), f);
    fclose(f);
  }
  f = fopen((base + ".shape").c_str(), "w");
  if (f) {
    fprintf(f, "%lld %d %d\n", rows, cols, ld);
    fclose(f);
  }
}

// Stage boundary: with the profile on, the device time since the previous boundary is recorded as
// class "stage:<what>" (launch count 1, no FLOPs); with KK_OPT_SYNC_EACH_STAGE the stream is
// synchronised so an error is reported against the stage that raised it.
void Engine::stage_sync(const char* what) {
  if (profile && stage_ev && !noalloc_active) {
    cudaEvent_t b = pool_event();
    KK_CUDA(cudaEventRecord(b, st));
    prof_pending.push_back({prof_class((std::string("stage:") + what).c_str()), stage_ev, b, 0.0, 0.0});
    stage_ev = b;
  }
  if (!sync_each) return;
  cudaError_t s = cudaStreamSynchronize(st);
  if (s != cudaSuccess) throw KKError(KK_ERR_CUDA, std::string(what) + ": " + cudaGetErrorString(s));
}

ConvArgs Engine::ca(const Conv& c) {
  ConvArgs a;
  memset(&a, 0, sizeof(a));
  a.w = c.w, a.bias = c.b, a.cin = c.cin, a.cout = c.cout, a.K = c.K, a.dil = c.dil, a.pad = c.pad,
  a.stride = c.stride;
  a.in_mode = IN_NOMASK;
  a.out_mode = OUT_STORE;
  a.oscale = 1.0f;
  a.nomask = negctl_nomask ? 1 : 0;
  return a;
}

void Engine::run_conv(const Conv& c, ConvArgs& a) {
  cudaEvent_t e0;
  prof_begin(&e0);
  const double flops = 2.0 * c.macs_per_row * a.L_out;
  // algorithmic bytes: f32 input rows read once, output rows written once (read too when
  // accumulated into), shortcut rows read once, weights once (bf16 image or f32)
  const bool res = a.out_mode == OUT_ADD || a.out_mode == OUT_PLUS;
  const bool tc_path = tc_route(c, a);
  const double in_rows = a.in_up2 ? (double)((a.L_in + 1) / 2) : (double)a.L_in;
  // bf16 window planes in or out: 2 bytes per element
  const double in_b = a.in_mode == IN_PRE ? 2.0 : (a.x_b ? 12.0 : 4.0),
               out_b = (a.out_mode == OUT_GELU_PRE || a.out_mode == OUT_STORE_BF) ? 2.0 : 4.0;
  const double out_bytes = out_b * (double)a.L_out * a.cout + (res ? 4.0 * a.L_out * a.cout : 0.0) +
                           (tc_path ? (double)c.tc.bytes : 4.0 * c.cin * c.cout * c.K);
  double bytes = in_b * in_rows * a.cin + out_bytes;
  if (tc_path) {
    unsigned long long* tr = nullptr;
    if (tc_trace_dir) {
      tr = ar.get<unsigned long long>(16);
      KK_CUDA(cudaMemsetAsync(tr, 0, 16 * sizeof(unsigned long long), st));
    }
    if (tc_pre(c, a) || (a.x_b && a.in_mode != IN_PRE)) {
      // several 128-channel output tiles share each input window (or the input is the mean of three
      // resblocks, formed here): transform the input once into bf16 window planes instead of once
      // per output tile
      auto mk = ar.mark();
      ConvArgs ap = a;
      ap.x_b = ap.x_c = nullptr;
      ap.pre_rows = PRE_PAD_FRONT + (long)a.L_in + PRE_PAD_BACK;
      void* xpre = ar.get<uint8_t>((size_t)((a.cin + 63) / 64) * 8 * ap.pre_rows * 16);
      check(launch_prologue_bf16(a, xpre, ap.pre_rows, st), "prologue_bf16");
      // the transform is its own (HBM-bound) kernel: profiled as its own class, so the conv class
      // is the tcgen05 kernel alone (which reads the bf16 planes)
      const double planes = 2.0 * (double)ap.pre_rows * ((a.cin + 63) / 64) * 64;
      prof_end(e0, "input_transform", 0.0, in_b * in_rows * a.cin + planes);
      prof_begin(&e0);
      bytes = 2.0 * in_rows * a.cin + out_bytes;
      ap.xpre = xpre;
      ap.in_mode = IN_PRE;
      ap.in_up2 = 0;
      check(tc_conv(ap, c.tc, err_flag, st, tr), "conv(tcgen05)");
      ar.rewind(mk);
    } else {
      check(tc_conv(a, c.tc, err_flag, st, tr), "conv(tcgen05)");
    }
    if (tr) {
      unsigned long long h[16];
      KK_CUDA(cudaStreamSynchronize(st));
      KK_CUDA(cudaMemcpy(h, tr, sizeof(h), cudaMemcpyDeviceToHost));
      FILE* f = fopen((std::string(tc_trace_dir) + "/tc_trace.txt").c_str(), "a");
      if (f) {
        fprintf(f, "K=%d dil=%d cin=%d cout=%d L=%d in=%d out=%d |", a.K, a.dil, a.cin, a.cout, a.L_out, a.in_mode,
                a.out_mode);
        for (int i = 0; i < 16; i++) fprintf(f, " %llu", h[i]);
        fprintf(f, "\n");
        fclose(f);
      }
    }
    if (prof_shapes) {
      char tag[96];
      snprintf(tag, sizeof(tag), "conv_tcgen05 k%d d%d %d>%d L%d in%d out%d st%d", a.K, a.dil, a.cin, a.cout, a.L_out,
               a.in_mode, a.out_mode, a.stat ? 1 : 0);
      prof_end(e0, tag, flops, bytes);
    } else {
      prof_end(e0, "conv_tcgen05", flops, bytes);
    }
  } else if (a.x_b) {  // the three-input mean outside the tensor-core route: form it first
    auto mk = ar.mark();
    const long n = (long)(a.in_up2 ? (a.L_in + 1) / 2 : a.L_in) * a.ldx;
    float* mean3 = ar.get<float>((size_t)n);
    check(launch_sum3(a.x, a.x_b, a.x_c, mean3, n, st), "sum3");
    ConvArgs a1 = a;
    a1.x = mean3, a1.x_b = a1.x_c = nullptr;
    run_conv(c, a1);
    ar.rewind(mk);
    return;
  } else if (rowproj_supported(a)) {  // projections to 1-4 channels: one warp per row
    check(launch_rowproj(a, st), "conv(row projection)");
    prof_end(e0, "rowproj", flops, bytes);
  } else {
    check(launch_conv_simt(a, st), "conv(simt)");
    prof_end(e0, "conv_simt", flops, bytes);
  }
}

bool Engine::tc_route(const Conv& c, const ConvArgs& a) const {
  return precision == KK_PRECISION_BF16 && tc_ok && c.tc.w && !c.simt_only && tc_supported(a, c.tc);
}

// Tensor-core layers whose input is first transformed into bf16 window planes (prologue kernel):
// several 128-channel output tiles share each input window, or a short kernel leaves the fused
// route's producers too little MMA time to hide behind.
bool Engine::tc_pre(const Conv& c, const ConvArgs& a) const {
  return (c.cout > TC_PRE_MIN_COUT || (c.cout == TC_PRE_MIN_COUT && c.K <= 3)) && a.in_mode != IN_PRE;
}

// Run a convolution and produce the AdaIN statistics of its output [L_out][cout] (ldy == cout):
// fused into the tensor-core epilogue when the layer runs there, else a separate stats pass.
void Engine::run_conv_stats(const Conv& c, ConvArgs& a, const Dom& dout, const ItemTab* items, int B, int max_len,
                            float** mean, float** rstd) {
  if (tc_route(c, a)) {
    double* part = ar.get<double>((size_t)2 * B * c.cout);
    KK_CUDA(cudaMemsetAsync(part, 0, sizeof(double) * 2 * B * c.cout, st));
    a.stat = part;
    a.dout = dout;
    run_conv(c, a);
    *mean = ar.get<float>((size_t)B * c.cout);
    *rstd = ar.get<float>((size_t)B * c.cout);
    check(launch_stats_from_sums(part, c.cout, items, B, dout.scale == 0 ? 1 : dout.scale, dout.plus1, *mean, *rstd,
                                 st),
          "stats_from_sums");
  } else {
    run_conv(c, a);
    stats(a.y, a.ldy, c.cout, dout, items, B, max_len, mean, rstd);
  }
}

void Engine::linear(const Conv& c, const float* x, int ldx, int rows, float* y, int ldy, int out_mode, const float* sc,
                    int ldsc) {
  ConvArgs a = ca(c);
  a.x = x, a.ldx = ldx, a.L_in = rows, a.y = y, a.ldy = ldy, a.L_out = rows, a.out_mode = out_mode, a.sc = sc,
  a.ldsc = ldsc;
  run_conv(c, a);
}

void Engine::stats(const float* x, int ldx, int C, const Dom& d, const ItemTab* items, int B, int max_len, float** mean,
                   float** rstd) {
  *mean = ar.get<float>((size_t)B * C);
  *rstd = ar.get<float>((size_t)B * C);
  double* part = ar.get<double>((size_t)2 * B * C);
  check(launch_stats(x, ldx, C, items, B, d.scale == 0 ? 1 : d.scale, d.plus1, max_len, part, *mean, *rstd, st),
        "stats");
  launches++;  // partial sums + finalisation: two kernels
}

void Engine::adain_args(ConvArgs& a, const AdaIN& n, const float* mean, const float* rstd, const float* gb, int ldgb,
                        int mode, float slope, const float* alpha) {
  a.in_mode = mode;
  a.mean = mean, a.rstd = rstd, a.nw = n.nw, a.nb = n.nb, a.gb = gb + n.off, a.ldgb = ldgb, a.slope = slope,
  a.alpha = alpha;
  a.coef = nullptr;
  if (precision == KK_PRECISION_BF16 && tc_ok) {
    float2* coef = ar.get<float2>((size_t)cur_B * n.c);
    check(launch_adain_coef(mean, rstd, n.nw, n.nb, gb + n.off, ldgb, cur_B, n.c, coef, st), "adain_coef");
    a.coef = coef;
  }
}

// AdainResBlk1d (src/gpu_batch.rs:103-135): y = (conv2(act(AdaIN2(conv1(pool?(act(AdaIN1(x))))))) + sc) / sqrt(2)
void Engine::resblk(const ResBlk& R, const float* x, int ldx, const Dom& din, const Dom& dout, float* y, int ldy,
                    const float* gb, int ldgb, const ItemTab* items, int B, int max_n) {
  auto mk = ar.mark();
  const int scale_in = din.scale, scale_out = dout.scale;
  float *m1, *r1, *m2, *r2;
  stats(x, ldx, R.din, din, items, B, max_n * scale_in, &m1, &r1);
  float* h = ar.get<float>((size_t)dout.L * R.dout);
  ConvArgs a = ca(R.c1);
  if (R.up) {
    const int ldp = ld16(R.din);
    float* p = ar.get<float>((size_t)dout.L * ldp);
    ConvArgs pro = ca(R.c1);
    pro.x = x, pro.ldx = ldx, pro.cin = R.din, pro.din = din;
    adain_args(pro, R.n1, m1, r1, gb, ldgb, IN_ADAIN_LEAKY, 0.2f, nullptr);
    check(launch_adain_pool(x, R.din, din.L, pro, R.pool_w, R.pool_b, p, ldp, st), "adain_pool");
    a.x = p, a.ldx = ldp, a.in_mode = IN_MASK, a.din = dout, a.L_in = dout.L;
  } else {
    a.x = x, a.ldx = ldx, a.din = din, a.L_in = din.L;
    adain_args(a, R.n1, m1, r1, gb, ldgb, IN_ADAIN_LEAKY, 0.2f, nullptr);
  }
  a.y = h, a.ldy = R.dout, a.L_out = dout.L;
  run_conv_stats(R.c1, a, dout, items, B, max_n * scale_out, &m2, &r2);
  const float* sc = x;
  int ldsc = ldx;
  if (R.has_sc) {
    float* s = ar.get<float>((size_t)dout.L * R.dout);
    ConvArgs c = ca(R.sc);
    c.x = x, c.ldx = ldx, c.in_mode = IN_MASK, c.in_up2 = R.up ? 1 : 0, c.din = dout, c.L_in = dout.L;
    c.y = s, c.ldy = R.dout, c.L_out = dout.L;
    run_conv(R.sc, c);
    sc = s, ldsc = R.dout;
  }
  ConvArgs b2 = ca(R.c2);
  b2.x = h, b2.ldx = R.dout, b2.din = dout, b2.L_in = dout.L;
  adain_args(b2, R.n2, m2, r2, gb, ldgb, IN_ADAIN_LEAKY, 0.2f, nullptr);
  b2.y = y, b2.ldy = ldy, b2.L_out = dout.L, b2.out_mode = OUT_PLUS, b2.sc = sc, b2.ldsc = ldsc;
  b2.oscale = 1.0f / sqrtf(2.0f);
  run_conv(R.c2, b2);
  ar.rewind(mk);
}

// AdaINResBlock1 with Snake (src/gpu_batch.rs:137-154): out = x_in + sum_i conv2_i(snake(AdaIN(conv1_i(snake(AdaIN(.))))))
void Engine::snake(const SnakeBlk& S, const float* xin, float* out, const Dom& d, const float* gb, int ldgb,
                   const ItemTab* items, int B, int max_n, const float* in_mean, const float* in_rstd) {
  auto mk = ar.mark();
  const int C = S.c;
  float* h = ar.get<float>((size_t)d.L * C);
  const float* cur = xin;
  const int max_len = max_n * d.scale + d.plus1;
  float *m1 = const_cast<float*>(in_mean), *r1 = const_cast<float*>(in_rstd);
  if (!m1) stats(xin, C, C, d, items, B, max_len, &m1, &r1);
  for (int i = 0; i < 3; i++) {
    float *m2, *r2;
    ConvArgs a = ca(S.c1[i]);
    a.x = cur, a.ldx = C, a.din = d, a.L_in = d.L, a.y = h, a.ldy = C, a.L_out = d.L;
    adain_args(a, S.a1[i], m1, r1, gb, ldgb, IN_ADAIN_SNAKE, 0.0f, S.al1[i]);
    run_conv_stats(S.c1[i], a, d, items, B, max_len, &m2, &r2);
    ConvArgs b = ca(S.c2[i]);
    b.x = h, b.ldx = C, b.din = d, b.L_in = d.L, b.y = out, b.ldy = C, b.L_out = d.L;
    adain_args(b, S.a2[i], m2, r2, gb, ldgb, IN_ADAIN_SNAKE, 0.0f, S.al2[i]);
    if (i == 0) {
      b.out_mode = OUT_PLUS, b.sc = xin, b.ldsc = C;
    } else {
      b.out_mode = OUT_ADD;
    }
    if (i < 2) {
      run_conv_stats(S.c2[i], b, d, items, B, max_len, &m1, &r1);  // statistics of the next sub-block's input
    } else {
      run_conv(S.c2[i], b);
    }
    cur = out;
  }
  ar.rewind(mk);
}

// One BiLSTM over row spans (src/gpu_batch.rs:157-175): gx = W_ih x + b_ih for both directions in
// one 1-tap conv, then the persistent recurrence.
void Engine::lstm(const Lstm& L, const float* x, int ldx, int rows, const std::vector<int>& start,
                  const std::vector<int>& len, float* out, int ldo) {
  auto mk = ar.mark();
  const int B = (int)start.size();
  float* gx = ar.get<float>((size_t)rows * 2048);
  linear(L.ih, x, ldx, rows, gx, 2048);
  std::vector<int> order(B);
  std::iota(order.begin(), order.end(), 0);
  std::stable_sort(order.begin(), order.end(), [&](int a, int b) { return len[a] > len[b]; });
  // groups of LSTM_IPG consecutive items of the longest-first order (one cluster per group and
  // direction; clusters are independent, so any number of groups is valid)
  const int IPG = LSTM_IPG;
  const int G = (B + IPG - 1) / IPG;
  const int Tmax = B ? len[order[0]] : 0;
  std::vector<int> gstart((size_t)G * IPG, 0), glen((size_t)G * IPG, 0), gact((size_t)G * std::max(Tmax, 1), 0);
  for (int r = 0; r < B; r++) {
    gstart[r] = start[order[r]];
    glen[r] = len[order[r]];
  }
  for (int g = 0; g < G; g++)
    for (int s2 = 0; s2 < Tmax; s2++) {
      int n = 0;
      while (n < IPG && glen[(size_t)g * IPG + n] > s2) n++;
      gact[(size_t)g * Tmax + s2] = n;
    }
  LstmArgs a;
  a.gx = gx, a.ldgx = 2048, a.whh = L.whh, a.bhh = L.bhh, a.out = out, a.ldo = ldo;
  a.gstart = upload(gstart.data(), gstart.size());
  a.glen = upload(glen.data(), glen.size());
  a.gact = upload(gact.data(), gact.size());
  a.G = G, a.IPG = IPG, a.Tmax = Tmax;
  a.tc = precision == KK_PRECISION_BF16 && tc_ok && L.f16_ok;
  a.err = err_flag;
  cudaEvent_t e0;
  prof_begin(&e0);
  check(launch_lstm(a, st), "lstm");
  long long steps = 0;
  for (int r = 0; r < B; r++) steps += len[r];
  prof_end(e0, "lstm_recurrence", 2.0 * 2 * 1024 * 256 * (double)steps);
  ar.rewind(mk);
}

// Decoder + generator on the frame layout (src/gpu_batch.rs:299-420). xcat0 [LN][514] holds asr
// in columns 0..511; f0 / nc are the 2N curves. Returns the audio buffer [600 LN].
float* Engine::decode_core(int B, const std::vector<ItemTab>& items_h, const ItemTab* items, const int* col_item_n,
                           int LN, float* xcat0, float* f0, float* nc, const float* gb_dec, int ldgb,
                           const uint64_t* seeds_d, const float* noise_d, const long long* noise_off_d) {
  int max_n = 0;
  for (auto& it : items_h) max_n = std::max(max_n, it.n);
  return decode_core(B, max_n, items, col_item_n, LN, xcat0, f0, nc, gb_dec, ldgb, seeds_d, noise_d, noise_off_d);
}

float* Engine::decode_core(int B, int max_n, const ItemTab* items, const int* col_item_n, int LN, float* xcat0,
                           float* f0, float* nc, const float* gb_dec, int ldgb, const uint64_t* seeds_d,
                           const float* noise_d, const long long* noise_off_d) {
  const Dom dN{col_item_n, LN, 1, 0, LN};
  const Dom d2{col_item_n, LN, 2, 0, 2 * LN};
  const Dom d20{col_item_n, LN, 20, 0, 20 * LN};
  const Dom d120{col_item_n, LN, 120, 1, 120 * LN + 1};
  const int L2 = 2 * LN, L20 = 20 * LN, L120 = 120 * LN + 1;
  // ---- decoder (pre-generator)
  float* catA = ar.get<float>((size_t)LN * CAT_LD);
  float* catB = ar.get<float>((size_t)LN * CAT_LD);
  CurveConv wf{m.f0conv_w, m.f0conv_b}, wn{m.nconv_w, m.nconv_b};
  check(launch_curve_conv(f0, nc, d2, LN, wf, wn, xcat0, X0_LD, 512, catA, CAT_LD, 1088, catB, CAT_LD, 1088, st),
        "curve_conv");
  {
    ConvArgs a = ca(m.asr_res);
    a.x = xcat0, a.ldx = X0_LD, a.in_mode = IN_MASK, a.din = dN, a.L_in = LN;
    a.y = catA + 1024, a.ldy = CAT_LD, a.L_out = LN;
    run_conv(m.asr_res, a);
    check(launch_copy_cols(catA, CAT_LD, 1024, catB, CAT_LD, 1024, LN, 64, st), "copy_cols");
  }
  dump("xcat0", xcat0, LN, 514, X0_LD);
  resblk(m.enc, xcat0, X0_LD, dN, dN, catA, CAT_LD, gb_dec, ldgb, items, B, max_n);
  dump("enc", catA, LN, 1090, CAT_LD);
  resblk(m.dec[0], catA, CAT_LD, dN, dN, catB, CAT_LD, gb_dec, ldgb, items, B, max_n);
  resblk(m.dec[1], catB, CAT_LD, dN, dN, catA, CAT_LD, gb_dec, ldgb, items, B, max_n);
  resblk(m.dec[2], catA, CAT_LD, dN, dN, catB, CAT_LD, gb_dec, ldgb, items, B, max_n);
  float* xd = ar.get<float>((size_t)L2 * 512);
  resblk(m.dec[3], catB, CAT_LD, dN, d2, xd, 512, gb_dec, ldgb, items, B, max_n);
  dump("xd", xd, L2, 512, 512);
  stage_sync("decoder");
  // ---- harmonic source + STFT (one launch each for the whole batch)
  float* pp = ar.get<float>((size_t)9 * L2);
  check(launch_sine_phase(f0, L2, items, B, pp, st), "sine_phase");
  float* har = ar.get<float>((size_t)600 * LN);
  check(launch_har_source(f0, pp, L2, items, col_item_n, LN, seeds_d, noise_d, noise_off_d, m.lw, m.lb, har, st),
        "har_source");
  // spectrum rows with 3 zero rows in front and 8 behind (the 6-frame-row view of noise_convs.0)
  float* spec_pad = ar.get<float>((size_t)(L120 + 11) * SPEC_LD);
  float* spec = spec_pad + 3 * SPEC_LD;
  KK_CUDA(cudaMemsetAsync(spec_pad, 0, sizeof(float) * 3 * SPEC_LD, st));
  KK_CUDA(cudaMemsetAsync(spec + (size_t)L120 * SPEC_LD, 0, sizeof(float) * 8 * SPEC_LD, st));
  check(launch_stft(har, items, d120, spec, SPEC_LD, st), "stft");
  dump("har", har, 600LL * LN, 1, 1);
  dump("spec", spec, L120, 22, SPEC_LD);
  stage_sync("source");
  // ---- generator stage 0 (2N -> 20N, C 256)
  float* y0 = ar.get<float>((size_t)L20 * 256);
  // BF16 mode on the tensor cores: stage 0's three resblock outputs stay alive and the input
  // transform of the stage-1 upsampling (the pre-transform route, which that layer takes anyway)
  // forms their mean, saving the mean pass over HBM. Stage 1 keeps the mean kernel: its consumer,
  // conv_post, runs on the fused route, and the pre-transform route with the three-input mean cost
  // it more than the mean kernel (measured: +2.8 ms against 2.2 ms). FP32 mode and stage dumps keep
  // the mean kernel for both stages
  const char* dump_dir = getenv("KK_DEBUG_DUMP_DIR");
  const bool fuse_mean = precision == KK_PRECISION_BF16 && tc_ok && !(dump_dir && *dump_dir);
  float* x1 = fuse_mean ? nullptr : ar.get<float>((size_t)L20 * 256);
  float* r1[3] = {nullptr, nullptr, nullptr};  // stage-0 resblock outputs (fuse_mean)
  if (fuse_mean)
    for (int j = 0; j < 3; j++) r1[j] = ar.get<float>((size_t)L20 * 256);
  {
    auto mk = ar.mark();
    float* xs = ar.get<float>((size_t)L20 * 256);
    float* xsr = ar.get<float>((size_t)L20 * 256);
    // statistics of the noise-conv output (the first AdaIN of noise_res) from the conv's epilogue
    float *xm, *xr;
    const int len20 = max_n * d20.scale + d20.plus1;
    if (m.noise0_rows.w) {
      // gap rows of the spectrum are zero (stft), so the 6-frame-row view needs no masking
      ConvArgs a = ca(m.noise0_rows);
      a.x = spec_pad, a.ldx = 6 * SPEC_LD, a.in_mode = IN_NOMASK, a.L_in = L20 + 1, a.y = xs, a.ldy = 256,
      a.L_out = L20;
      run_conv_stats(m.noise0_rows, a, d20, items, B, len20, &xm, &xr);
    } else {
      ConvArgs a = ca(m.noise0);
      a.x = spec, a.ldx = SPEC_LD, a.in_mode = IN_MASK, a.din = d120, a.L_in = L120, a.y = xs, a.ldy = 256,
      a.L_out = L20;
      run_conv_stats(m.noise0, a, d20, items, B, len20, &xm, &xr);
    }
    snake(m.noise_res[0], xs, xsr, d20, gb_dec, ldgb, items, B, max_n, xm, xr);
    ConvArgs u = ca(m.ups[0]);
    u.x = xd, u.ldx = 512, u.in_mode = IN_LEAKY_MASK, u.slope = 0.1f, u.din = d2, u.L_in = L2;
    u.y = y0, u.ldy = 2560, u.L_out = L2, u.out_mode = OUT_PLUS, u.sc = xsr, u.ldsc = 2560;
    run_conv(m.ups[0], u);
    dump("xs0", xs, L20, 256, 256);
    dump("xsr0", xsr, L20, 256, 256);
    dump("y0", y0, L20, 256, 256);
    ar.rewind(mk);
    float* r[3];
    float *ym, *yr;  // statistics of y0, shared by the three parallel resblocks
    stats(y0, 256, 256, d20, items, B, max_n * d20.scale + d20.plus1, &ym, &yr);
    for (int j = 0; j < 3; j++) {
      r[j] = fuse_mean ? r1[j] : ar.get<float>((size_t)L20 * 256);
      snake(m.rb[j], y0, r[j], d20, gb_dec, ldgb, items, B, max_n, ym, yr);
    }
    if (!fuse_mean) {
      cudaEvent_t e0;
      prof_begin(&e0);
      check(launch_sum3(r[0], r[1], r[2], x1, (long)L20 * 256, st), "sum3");
      prof_end(e0, "resblock_mean", 0.0, 16.0 * (double)L20 * 256);
    }
    dump("r0_0", r[0], L20, 256, 256);
    dump("x1", x1, L20, 256, 256);
    ar.rewind(mk);
  }
  stage_sync("generator stage 0");
  // ---- generator stage 1 (20N -> 120N + 1, C 128)
  float* y1 = ar.get<float>((size_t)L120 * 128);
  float* x2 = ar.get<float>((size_t)L120 * 128);
  // BF16 mode: the AdaIN statistics of y1 come out of the reflection-pad pass that writes it
  // (plain f32 partial sums, as the tensor-core epilogues form theirs) instead of a second pass
  const bool y1_fused_stats = precision == KK_PRECISION_BF16 && tc_ok;
  float *ym1 = nullptr, *yr1 = nullptr;
  double* part1 = nullptr;
  if (y1_fused_stats) {
    part1 = ar.get<double>((size_t)2 * B * 128);
    ym1 = ar.get<float>((size_t)B * 128);
    yr1 = ar.get<float>((size_t)B * 128);
  }
  {
    auto mk = ar.mark();
    float* xs = ar.get<float>((size_t)L120 * 128);
    float* xsr = ar.get<float>((size_t)L120 * 128);
    ConvArgs a = ca(m.noise1);
    a.x = spec, a.ldx = SPEC_LD, a.in_mode = IN_MASK, a.din = d120, a.L_in = L120, a.y = xs, a.ldy = 128,
    a.L_out = L120;
    float *xm, *xr;  // statistics of the noise-conv output from the conv's epilogue
    run_conv_stats(m.noise1, a, d120, items, B, max_n * d120.scale + d120.plus1, &xm, &xr);
    snake(m.noise_res[1], xs, xsr, d120, gb_dec, ldgb, items, B, max_n, xm, xr);
    float* u1 = xs;  // noise-conv output no longer needed
    ConvArgs u = ca(m.ups[1]);
    u.x = fuse_mean ? r1[0] : x1, u.ldx = 256, u.in_mode = IN_LEAKY_MASK, u.slope = 0.1f, u.din = d20, u.L_in = L20;
    if (fuse_mean) u.x_b = r1[1], u.x_c = r1[2];
    u.y = u1, u.ldy = 768, u.L_out = L20;
    run_conv(m.ups[1], u);
    if (y1_fused_stats) {
      KK_CUDA(cudaMemsetAsync(part1, 0, sizeof(double) * 2 * B * 128, st));
      check(launch_reflect_add_stats(u1, xsr, items, d120, y1, part1, st), "reflect_add_stats");
      check(launch_stats_from_sums(part1, 128, items, B, d120.scale, d120.plus1, ym1, yr1, st), "stats_from_sums");
    } else {
      check(launch_reflect_add(u1, xsr, 128, items, d120, y1, st), "reflect_add");
    }
    dump("xsr1", xsr, L120, 128, 128);
    dump("y1", y1, L120, 128, 128);
    ar.rewind(mk);
    float* r[3];
    float *ym, *yr;  // statistics of y1, shared by the three parallel resblocks
    if (y1_fused_stats)
      ym = ym1, yr = yr1;
    else
      stats(y1, 128, 128, d120, items, B, max_n * d120.scale + d120.plus1, &ym, &yr);
    for (int j = 0; j < 3; j++) {
      r[j] = ar.get<float>((size_t)L120 * 128);
      snake(m.rb[3 + j], y1, r[j], d120, gb_dec, ldgb, items, B, max_n, ym, yr);
    }
    {
      cudaEvent_t e0;
      prof_begin(&e0);
      check(launch_sum3(r[0], r[1], r[2], x2, (long)L120 * 128, st), "sum3");
      prof_end(e0, "resblock_mean", 0.0, 16.0 * (double)L120 * 128);
    }
    dump("x2", x2, L120, 128, 128);
    ar.rewind(mk);
  }
  stage_sync("generator stage 1");
  // ---- conv_post + iSTFT
  float* post = ar.get<float>((size_t)L120 * POST_LD);
  {
    ConvArgs a = ca(m.post);
    a.x = x2, a.ldx = 128, a.in_mode = IN_LEAKY_MASK, a.slope = 0.01f, a.din = d120, a.L_in = L120;
    a.y = post, a.ldy = POST_LD, a.L_out = L120;
    run_conv(m.post, a);
  }
  float* audio = ar.get<float>((size_t)600 * LN);
  check(launch_istft(post, POST_LD, items, d120, col_item_n, LN, audio, st), "istft");
  times_compute_end();
  dump("post", post, L120, 22, POST_LD);
  dump("audio", audio, 600LL * LN, 1, 1);
  stage_sync("istft");
  return audio;
}

void Engine::finish_audio(float* audio_d, int LN, const std::vector<ItemTab>& items_h, const int* col_item_n,
                          bool pcm16) {
  const size_t n = (size_t)600 * LN;
  out_off.clear();
  out_len.clear();
  for (auto& it : items_h) {
    out_off.push_back(600LL * it.a);
    out_len.push_back(600LL * it.n);
  }
  int errh = 0;
  unsigned long long* clip_h = nullptr;
  if (!keep_audio_dev && pcm16 && pcm16_out) {
    // PCM_16 on the device: half the bytes cross PCIe
    if (audio_host16_cap < n) {
      if (audio_host16) cudaFreeHost(audio_host16);
      audio_host16 = nullptr;
      audio_host16_cap = 0;
      if (cudaHostAlloc(&audio_host16, n * sizeof(int16_t), cudaHostAllocDefault) != cudaSuccess) {
        cudaGetLastError();
        audio_host16 = nullptr;
        throw KKError(KK_ERR_OOM, "pinned audio buffer");
      }
      audio_host16_cap = n;
    }
    const int B = (int)items_h.size();
    int16_t* q = ar.get<int16_t>(n);
    unsigned long long* clip = ar.get<unsigned long long>((size_t)std::max(B, 1));
    KK_CUDA(cudaMemsetAsync(clip, 0, sizeof(unsigned long long) * std::max(B, 1), st));
    check(launch_pcm16(audio_d, (long)n, col_item_n, q, clip, st), "pcm16");
    KK_CUDA(cudaMemcpyAsync(audio_host16, q, n * sizeof(int16_t), cudaMemcpyDeviceToHost, st));
    clip_h = (unsigned long long*)pin.alloc(sizeof(unsigned long long) * std::max(B, 1));
    KK_CUDA(cudaMemcpyAsync(clip_h, clip, sizeof(unsigned long long) * std::max(B, 1), cudaMemcpyDeviceToHost, st));
    d2h_bytes += (double)(n * sizeof(int16_t));
  } else if (!keep_audio_dev) {
    if (audio_host_cap < n) {
      if (audio_host) cudaFreeHost(audio_host);
      audio_host = nullptr;
      audio_host_cap = 0;
      if (cudaHostAlloc(&audio_host, n * sizeof(float), cudaHostAllocDefault) != cudaSuccess) {
        cudaGetLastError();
        audio_host = nullptr;
        throw KKError(KK_ERR_OOM, "pinned audio buffer");
      }
      audio_host_cap = n;
    }
    KK_CUDA(cudaMemcpyAsync(audio_host, audio_d, n * sizeof(float), cudaMemcpyDeviceToHost, st));
    d2h_bytes += (double)(n * sizeof(float));
  }
  int* eh = (int*)pin.alloc(sizeof(int));
  KK_CUDA(cudaMemcpyAsync(eh, err_flag, sizeof(int), cudaMemcpyDeviceToHost, st));
  KK_CUDA(cudaEventRecord(ev[3], st));
  KK_CUDA(cudaStreamSynchronize(st));
  errh = *eh;
  out_clipped.assign(items_h.size(), 0);
  if (clip_h)
    for (size_t b = 0; b < items_h.size(); b++) out_clipped[b] = (long long)clip_h[b];
  if (errh) throw KKError(KK_ERR_TIMEOUT, wait_error(errh));
  float t_all = 0, t_comp = 0;
  KK_CUDA(cudaEventElapsedTime(&t_all, ev[0], ev[3]));
  KK_CUDA(cudaEventElapsedTime(&t_comp, ev[1], ev[2]));
  last_times[0] = t_all, last_times[1] = t_comp, last_times[2] = h2d_bytes, last_times[3] = d2h_bytes;
  prof_collect();
}

void Engine::upload_noise(int B, const std::vector<ItemTab>& items_h, const float* const* noise, float** noise_d,
                          long long** noise_off_d) {
  std::vector<long long> off(B, -1);
  long long tot = 0;
  for (int b = 0; b < B; b++)
    if (noise[b]) off[b] = tot, tot += 600LL * 9 * items_h[b].n;
  float* d = ar.get<float>((size_t)std::max(tot, 1LL));
  for (int b = 0; b < B; b++) {
    if (!noise[b]) continue;
    const size_t bytes = sizeof(float) * 600 * 9 * (size_t)items_h[b].n;
    void* s = pin.alloc(bytes);
    memcpy(s, noise[b], bytes);
    KK_CUDA(cudaMemcpyAsync(d + off[b], s, bytes, cudaMemcpyHostToDevice, st));
    h2d_bytes += (double)bytes;
  }
  *noise_d = d;
  *noise_off_d = upload(off.data(), B);
}

void Engine::forward(int B, const int64_t* ids, const int32_t* ids_len, const float* ref_s, const float* speed,
                     const uint64_t* seeds, const float* const* noise, const int64_t* noise_len,
                     const float* rand_ini, const int64_t* forced, int64_t* dur_out, int64_t* nsamp_out) {
  KK_REQUIRE(B > 0, "empty batch");
  KK_REQUIRE(ids && ids_len && ref_s && speed, "null input pointer");
  KK_REQUIRE(!noise || noise_len, "replayed noise without its lengths");
  // rand_ini of ItemNoise::Fixed is validated and otherwise unused: the reference adds it to the rad
  // curve at sample 0 only, which the linear x1/300 downsample of the phase never reads (its first
  // source position is 149.5), so it cannot change the output
  if (rand_ini)
    for (int i = 0; i < 9 * B; i++) KK_REQUIRE(std::isfinite(rand_ini[i]), "rand_ini must be finite");
  long long total_ids = 0;
  for (int b = 0; b < B; b++) {
    KK_REQUIRE(ids_len[b] >= 2 && ids_len[b] <= 512, "input_ids length outside [2, 512]");
    KK_REQUIRE(std::isfinite(speed[b]) && speed[b] > 0.0f, "speed must be positive and finite");
    total_ids += ids_len[b];
  }
  for (long long i = 0; i < total_ids; i++) KK_REQUIRE(ids[i] >= 0 && ids[i] < 178, "token id out of range");
  if (forced) {
    long long o = 0;
    for (int b = 0; b < B; b++) {
      long long s = 0;
      for (int i = 0; i < ids_len[b]; i++) {
        KK_REQUIRE(forced[o + i] >= 0 && forced[o + i] <= (1 << 20), "forced duration out of range");
        s += forced[o + i];
      }
      KK_REQUIRE(s >= 1, "forced durations of an item sum to zero");
      o += ids_len[b];
    }
  }
  KK_CUDA(cudaSetDevice(dev));
  ar.reset();
  ar.set_poison(gap_canary ? st : nullptr);
  pin.reset();
  prof_pending.clear();
  ev_used = 0;
  times_begin();
  KK_CUDA(cudaMemsetAsync(err_flag, 0, sizeof(int), st));
  // ---- token layout (src/gpu_batch.rs:189-213)
  std::vector<ItemTab> items_h(B);
  int LT = 0;
  last_tokens = 0;
  for (int b = 0; b < B; b++) {
    items_h[b] = {LT, ids_len[b], 0, 0};
    LT += ids_len[b] + GAP_T;
    last_tokens += ids_len[b];
  }
  LT = std::max(LT, MIN_LAYOUT_ROWS);
  std::vector<int> row_item_h(LT, -1), ids_h(LT, 0);
  {
    long long o = 0;
    for (int b = 0; b < B; b++) {
      for (int i = 0; i < ids_len[b]; i++) {
        row_item_h[items_h[b].tok_start + i] = b;
        ids_h[items_h[b].tok_start + i] = (int)ids[o + i];
      }
      o += ids_len[b];
    }
  }
  std::vector<float> sdec_h((size_t)B * 128), spro_h((size_t)B * 128);
  for (int b = 0; b < B; b++) {
    memcpy(&sdec_h[(size_t)b * 128], ref_s + (size_t)b * 256, 128 * sizeof(float));
    memcpy(&spro_h[(size_t)b * 128], ref_s + (size_t)b * 256 + 128, 128 * sizeof(float));
  }
  int* ids_d = upload(ids_h.data(), LT);
  int* row_item_d = upload(row_item_h.data(), LT);
  ItemTab* items_d = upload(items_h.data(), B);
  float* sdec_d = upload(sdec_h.data(), sdec_h.size());
  float* spro_d = upload(spro_h.data(), spro_h.size());
  float* speed_d = upload(speed, B);
  times_compute_begin();
  const Dom dT{row_item_d, 0, 0, 0, LT};
  cur_B = B;
  std::vector<int> tstart(B), tlen(B);
  for (int b = 0; b < B; b++) tstart[b] = items_h[b].tok_start, tlen[b] = items_h[b].tok_len;
  // ---- fused style projections (every AdaIN / AdaLN gamma|beta of the batch)
  const int wdec = m.fc_dec.cout, wpro = m.fc_pro.cout;
  float* gb_dec = ar.get<float>((size_t)B * wdec);
  float* gb_pro = ar.get<float>((size_t)B * wpro);
  linear(m.fc_dec, sdec_d, 128, B, gb_dec, wdec);
  linear(m.fc_pro, spro_d, 128, B, gb_pro, wpro);
  // ---- ALBERT (src/gpu_batch.rs:423-455)
  float* x640 = ar.get<float>((size_t)LT * 640);
  {
    auto mk = ar.mark();
    float* emb = ar.get<float>((size_t)LT * 128);
    check(launch_albert_embed(ids_d, row_item_d, items_d, LT, m.word, m.pos, m.tt0, m.emb_g, m.emb_b, emb, st),
          "albert_embed");
    float* h = ar.get<float>((size_t)LT * 768);
    float* qkv = ar.get<float>((size_t)LT * 2304);
    float* ctx = ar.get<float>((size_t)LT * 768);
    float* a = ar.get<float>((size_t)LT * 768);
    // BF16 mode on the tensor cores: every ALBERT linear reads its input as bf16 window planes
    // written by the stage before it (the attention for the output projection, the LayerNorms for
    // the QKV and FFN projections, the FFN's GELU epilogue for the down projection), so no f32
    // activation makes a round trip through HBM only to be transformed again; the QKV projection
    // writes bf16 rows, the attention's operand precision (rounded exactly as the attention would
    // round f32 rows)
    float* f = nullptr;
    const long pre_rows = PRE_PAD_FRONT + (long)LT + PRE_PAD_BACK;
    const size_t planes768 = (size_t)(768 / 64) * 8 * pre_rows * 16;
    void *hpre = nullptr, *ctxpre = nullptr, *apre = nullptr, *fpre = nullptr;
    bool planes = false;
    // tensor-core attention (BF16 mode); KK_OPT_ATTENTION_F32 keeps the fp32 kernel for comparisons
    const bool attn_tc = precision == KK_PRECISION_BF16 && tc_ok && !attn_f32;
    auto pre_args = [&](const Conv& c, const void* xp, float* y, int ldy, int out_mode, const float* sc, void* yp) {
      ConvArgs t = ca(c);
      t.in_mode = IN_PRE, t.xpre = xp, t.pre_rows = pre_rows, t.L_in = LT;
      t.y = y, t.ldy = ldy, t.L_out = LT, t.out_mode = out_mode, t.sc = sc, t.ldsc = 768;
      t.ypre = yp, t.ypre_rows = pre_rows;
      return t;
    };
    if (precision == KK_PRECISION_BF16 && tc_ok) {
      hpre = ar.get<uint8_t>(planes768);
      ctxpre = ar.get<uint8_t>(planes768);
      apre = ar.get<uint8_t>(planes768);
      fpre = ar.get<uint8_t>((size_t)(2048 / 64) * 8 * pre_rows * 16);
      ConvArgs t0 = pre_args(m.qkv, hpre, qkv, 2304, OUT_STORE_BF, nullptr, nullptr);
      ConvArgs t1 = pre_args(m.dense, ctxpre, a, 768, OUT_PLUS, h, nullptr);
      ConvArgs t2 = pre_args(m.ffn, apre, nullptr, 0, OUT_GELU_PRE, nullptr, fpre);
      ConvArgs t3 = pre_args(m.ffn_out, fpre, h, 768, OUT_PLUS, a, nullptr);
      ConvArgs t00 = ca(m.qkv);  // the first layer: f32 rows from map_in, through the pre-transform route
      t00.x = h, t00.ldx = 768, t00.L_in = LT, t00.y = qkv, t00.ldy = 2304, t00.L_out = LT, t00.out_mode = OUT_STORE_BF;
      planes = attn_tc && tc_route(m.qkv, t0) && tc_route(m.qkv, t00) && tc_pre(m.qkv, t00) &&
               tc_route(m.dense, t1) && tc_route(m.ffn, t2) && tc_route(m.ffn_out, t3);
    }
    if (!planes) f = ar.get<float>((size_t)LT * 2048);
    linear(m.map_in, emb, 128, LT, h, 768);
    int max_t = 0;
    for (int b = 0; b < B; b++) max_t = std::max(max_t, ids_len[b]);
    // tensor-core attention: (item, first query row) per 128-query tile, in length buckets
    int n_work[3] = {0, 0, 0};
    const int2* work_d = nullptr;
    if (attn_tc) {
      std::vector<int2> wl[3];
      for (int b = 0; b < B; b++) {
        const int T = ids_len[b];
        const int k = T <= 128 ? 0 : (T <= 256 ? 1 : 2);
        for (int q0 = 0; q0 < T; q0 += 128) wl[k].push_back(make_int2(b, q0));
      }
      std::vector<int2> all;
      for (int k = 0; k < 3; k++) {
        n_work[k] = (int)wl[k].size();
        all.insert(all.end(), wl[k].begin(), wl[k].end());
      }
      work_d = upload(all.data(), all.size());
    }
    for (int layer = 0; layer < 12; layer++) {
      if (planes && layer > 0) {
        ConvArgs t = pre_args(m.qkv, hpre, qkv, 2304, OUT_STORE_BF, nullptr, nullptr);
        run_conv(m.qkv, t);
      } else if (planes) {
        ConvArgs t = ca(m.qkv);
        t.x = h, t.ldx = 768, t.L_in = LT, t.y = qkv, t.ldy = 2304, t.L_out = LT, t.out_mode = OUT_STORE_BF;
        run_conv(m.qkv, t);
      } else {
        linear(m.qkv, h, 768, LT, qkv, 2304);  // the first layer's input comes from map_in
      }
      cudaEvent_t e0;
      prof_begin(&e0);
      if (attn_tc) {
        check(launch_attention_tc(qkv, 2304, planes, items_d, work_d, n_work, ctx, 768, err_flag, st,
                                  planes ? ctxpre : nullptr, pre_rows),
              "attention(tcgen05)");
        launches += (n_work[0] > 0) + (n_work[1] > 0) + (n_work[2] > 0) - 1;  // one kernel per non-empty bucket
      } else
        check(launch_attention_f32(qkv, 2304, items_d, B, max_t, ctx, 768, st), "attention");
      double af = 0;
      for (int b = 0; b < B; b++) af += 4.0 * 12 * 64 * (double)ids_len[b] * ids_len[b];
      prof_end(e0, "attention", af);
      if (planes) {
        ConvArgs t1 = pre_args(m.dense, ctxpre, a, 768, OUT_PLUS, h, nullptr);
        run_conv(m.dense, t1);
      } else {
        linear(m.dense, ctx, 768, LT, a, 768, OUT_PLUS, h, 768);
      }
      check(launch_ln_rows(a, 768, LT, 768, m.attn_g, m.attn_b, 1e-12f, 0, 0.0f, nullptr, nullptr, 0, nullptr, 0, a,
                           768, st, planes ? apre : nullptr, pre_rows),
            "ln");
      if (planes) {
        ConvArgs t2 = pre_args(m.ffn, apre, nullptr, 0, OUT_GELU_PRE, nullptr, fpre);
        run_conv(m.ffn, t2);
        ConvArgs t3 = pre_args(m.ffn_out, fpre, h, 768, OUT_PLUS, a, nullptr);
        run_conv(m.ffn_out, t3);
      } else {
        linear(m.ffn, a, 768, LT, f, 2048, OUT_GELU);
        linear(m.ffn_out, f, 2048, LT, h, 768, OUT_PLUS, a, 768);
      }
      check(launch_ln_rows(h, 768, LT, 768, m.full_g, m.full_b, 1e-12f, 0, 0.0f, nullptr, nullptr, 0, nullptr, 0, h,
                           768, st, planes && layer < 11 ? hpre : nullptr, pre_rows),
            "ln");
    }
    // bert_encoder -> d_en, then [d_en | s_pro] (src/gpu_batch.rs:223-231)
    linear(m.bert_enc, h, 768, LT, x640, 640);
    check(launch_cat_style(row_item_d, LT, 512, spro_d, 128, x640, 640, st), "cat_style");
    dump("bert", h, LT, 768, 768);
    dump("d_en", x640, LT, 640, 640);
    ar.rewind(mk);
  }
  stage_sync("albert");
  // ---- duration encoder + predictor LSTM + duration logits (src/gpu_batch.rs:224-248)
  int* dur_d = ar.get<int>(LT);
  float* q_d = ar.get<float>(LT);
  {
    auto mk = ar.mark();
    float* hl = ar.get<float>((size_t)LT * 512);
    for (int i = 0; i < 3; i++) {
      lstm(m.dur_lstm[i], x640, 640, LT, tstart, tlen, hl, 512);
      check(launch_ln_rows(hl, 512, LT, 512, nullptr, nullptr, 1e-5f, 2, 0.0f, row_item_d, gb_pro + m.adaln_off[i],
                           wpro, spro_d, 128, x640, 640, st),
            "adaln");
    }
    lstm(m.pred_lstm, x640, 640, LT, tstart, tlen, hl, 512);
    float* logits = ar.get<float>((size_t)LT * 50);
    linear(m.dur_proj, hl, 512, LT, logits, 50);
    check(launch_durations(logits, 50, row_item_d, speed_d, LT, dur_d, q_d, st), "durations");
    dump("x640", x640, LT, 640, 640);
    dump("logits", logits, LT, 50, 50);
    ar.rewind(mk);
  }
  stage_sync("durations");
  // ---- durations to the host: the one mid-forward synchronisation (src/gpu_batch.rs:243-248)
  std::vector<int> dur_h(LT, 0);
  if (forced) {
    long long o = 0;
    for (int b = 0; b < B; b++) {
      for (int i = 0; i < ids_len[b]; i++) dur_h[items_h[b].tok_start + i] = (int)forced[o + i];
      o += ids_len[b];
    }
  } else {
    int* dh = (int*)pin.alloc(sizeof(int) * LT);
    int* eh = (int*)pin.alloc(sizeof(int));
    KK_CUDA(cudaMemcpyAsync(dh, dur_d, sizeof(int) * LT, cudaMemcpyDeviceToHost, st));
    KK_CUDA(cudaMemcpyAsync(eh, err_flag, sizeof(int), cudaMemcpyDeviceToHost, st));
    KK_CUDA(cudaStreamSynchronize(st));
    if (*eh) throw KKError(KK_ERR_TIMEOUT, wait_error(*eh));
    memcpy(dur_h.data(), dh, sizeof(int) * LT);
  }
  if (dur_out) {
    long long o = 0;
    for (int b = 0; b < B; b++) {
      for (int i = 0; i < ids_len[b]; i++) dur_out[o + i] = dur_h[items_h[b].tok_start + i];
      o += ids_len[b];
    }
  }
  // ---- frame layout (src/gpu_batch.rs:250-279)
  int LN = 0;
  for (int b = 0; b < B; b++) {
    long long n = 0;
    for (int i = 0; i < ids_len[b]; i++) n += dur_h[items_h[b].tok_start + i];
    KK_REQUIRE(n >= 1 && n < (1 << 22), "item frame count out of range");
    items_h[b].a = LN;
    items_h[b].n = (int)n;
    LN += (int)n + GAP_N;
  }
  LN = std::max(LN, MIN_LAYOUT_ROWS);
  last_frames = 0;
  for (int b = 0; b < B; b++) last_frames += items_h[b].n;
  if (noise)
    for (int b = 0; b < B; b++)
      KK_REQUIRE(!noise[b] || noise_len[b] == 600LL * 9 * items_h[b].n,
                 "fixed noise size mismatch for item " + std::to_string(b) + " (needs 600 * 9 * " +
                     std::to_string(items_h[b].n) + " draws)");
  if (nsamp_out)
    for (int b = 0; b < B; b++) nsamp_out[b] = 600LL * items_h[b].n;
  std::vector<int> col_item_h(LN, -1), src_row_h(LN, -1);
  for (int b = 0; b < B; b++) {
    int f = items_h[b].a;
    for (int i = 0; i < ids_len[b]; i++)
      for (int k = 0; k < dur_h[items_h[b].tok_start + i]; k++) {
        col_item_h[f] = b;
        src_row_h[f] = items_h[b].tok_start + i;
        f++;
      }
  }
  items_d = upload(items_h.data(), B);
  int* col_item_d = upload(col_item_h.data(), LN);
  int* src_row_d = upload(src_row_h.data(), LN);
  stage_sync("frame layout");  // durations read-back, host layout build and upload
  const Dom dN{col_item_d, LN, 1, 0, LN};
  const Dom d2{col_item_d, LN, 2, 0, 2 * LN};
  std::vector<int> fstart(B), flen(B);
  int max_n = 0;
  for (int b = 0; b < B; b++) fstart[b] = items_h[b].a, flen[b] = items_h[b].n, max_n = std::max(max_n, flen[b]);
  // ---- F0 / N predictor (src/gpu_batch.rs:281-292)
  float* f0 = ar.get<float>((size_t)2 * LN);
  float* nc = ar.get<float>((size_t)2 * LN);
  {
    auto mk = ar.mark();
    float* en = ar.get<float>((size_t)LN * 640);
    check(launch_gather_rows(x640, 640, src_row_d, LN, 640, en, 640, st), "gather_rows");
    float* sh = ar.get<float>((size_t)LN * 512);
    lstm(m.shared, en, 640, LN, fstart, flen, sh, 512);
    dump("sh", sh, LN, 512, 512);
    float* h1 = ar.get<float>((size_t)LN * 512);
    float* h2 = ar.get<float>((size_t)2 * LN * 256);
    float* h3 = ar.get<float>((size_t)2 * LN * 256);
    for (int s = 0; s < 2; s++) {
      const ResBlk* blk = s == 0 ? m.f0 : m.nn;
      resblk(blk[0], sh, 512, dN, dN, h1, 512, gb_pro, wpro, items_d, B, max_n);
      resblk(blk[1], h1, 512, dN, d2, h2, 256, gb_pro, wpro, items_d, B, max_n);
      resblk(blk[2], h2, 256, d2, d2, h3, 256, gb_pro, wpro, items_d, B, max_n);
      const Conv& proj = s == 0 ? m.f0_proj : m.n_proj;
      ConvArgs a = ca(proj);
      a.x = h3, a.ldx = 256, a.in_mode = IN_MASK, a.din = d2, a.L_in = 2 * LN;
      a.y = s == 0 ? f0 : nc, a.ldy = 1, a.L_out = 2 * LN;
      run_conv(proj, a);
    }
    ar.rewind(mk);
  }
  dump("f0", f0, 2LL * LN, 1, 1);
  dump("nc", nc, 2LL * LN, 1, 1);
  stage_sync("f0n");
  // ---- text encoder (src/gpu_batch.rs:457-481) and alignment of its output (asr)
  float* xcat0 = ar.get<float>((size_t)LN * X0_LD);
  {
    auto mk = ar.mark();
    float* e = ar.get<float>((size_t)LT * 512);
    float* y = ar.get<float>((size_t)LT * 512);
    check(launch_embed_rows(ids_d, row_item_d, LT, m.te_emb, 512, e, st), "embed");
    float* cur = e;
    float* nxt = y;
    for (int i = 0; i < 3; i++) {
      ConvArgs a = ca(m.te_cnn[i]);
      a.x = cur, a.ldx = 512, a.in_mode = IN_MASK, a.din = dT, a.L_in = LT, a.y = nxt, a.ldy = 512, a.L_out = LT;
      run_conv(m.te_cnn[i], a);
      check(launch_ln_rows(nxt, 512, LT, 512, m.te_g[i], m.te_b[i], 1e-5f, 1, 0.2f, nullptr, nullptr, 0, nullptr, 0,
                           nxt, 512, st),
            "ln");
      std::swap(cur, nxt);
    }
    float* t_en = nxt;
    lstm(m.te_lstm, cur, 512, LT, tstart, tlen, t_en, 512);
    dump("t_en", t_en, LT, 512, 512);
    check(launch_gather_rows(t_en, 512, src_row_d, LN, 512, xcat0, X0_LD, st), "gather_rows");
    ar.rewind(mk);
  }
  stage_sync("text encoder");
  // ---- noise inputs (ItemNoise per item, src/gpu_batch.rs:325-340)
  uint64_t* seeds_d = nullptr;
  if (seeds) seeds_d = upload(seeds, B);
  float* noise_d = nullptr;
  long long* noise_off_d = nullptr;
  if (noise) upload_noise(B, items_h, noise, &noise_d, &noise_off_d);
  float* audio = decode_core(B, items_h, items_d, col_item_d, LN, xcat0, f0, nc, gb_dec, wdec, seeds_d, noise_d,
                             noise_off_d);
  finish_audio(audio, LN, items_h, col_item_d, true);
}

void Engine::decode(int B, const int32_t* n_frames, const float* asr, const float* f0_in, const float* n_in,
                    const float* s_dec, const uint64_t* seeds, const float* noise, float* audio_out) {
  KK_REQUIRE(B > 0, "empty batch");
  KK_REQUIRE(n_frames && asr && f0_in && n_in && s_dec, "null input pointer");
  std::vector<ItemTab> items_h(B);
  int LN = 0;
  long long tot = 0;
  for (int b = 0; b < B; b++) {
    KK_REQUIRE(n_frames[b] >= 1 && n_frames[b] < (1 << 22), "frame count out of range");
    items_h[b] = {0, 0, LN, n_frames[b]};
    LN += n_frames[b] + GAP_N;
    tot += n_frames[b];
  }
  LN = std::max(LN, MIN_LAYOUT_ROWS);
  last_tokens = 0;
  last_frames = tot;
  KK_CUDA(cudaSetDevice(dev));
  ar.reset();
  ar.set_poison(gap_canary ? st : nullptr);
  pin.reset();
  prof_pending.clear();
  ev_used = 0;
  times_begin();
  KK_CUDA(cudaMemsetAsync(err_flag, 0, sizeof(int), st));
  std::vector<int> col_item_h(LN, -1), tab1(LN, -1), tab2(2 * LN, -1);
  long long r = 0;
  for (int b = 0; b < B; b++) {
    for (int i = 0; i < items_h[b].n; i++) {
      col_item_h[items_h[b].a + i] = b;
      tab1[items_h[b].a + i] = (int)(r + i);
    }
    for (int i = 0; i < 2 * items_h[b].n; i++) tab2[2 * items_h[b].a + i] = (int)(2 * r + i);
    r += items_h[b].n;
  }
  ItemTab* items_d = upload(items_h.data(), B);
  int* col_item_d = upload(col_item_h.data(), LN);
  int* tab1_d = upload(tab1.data(), LN);
  int* tab2_d = upload(tab2.data(), 2 * LN);
  float* asr_d = upload(asr, (size_t)tot * 512);
  float* f0c_d = upload(f0_in, (size_t)2 * tot);
  float* nc_d = upload(n_in, (size_t)2 * tot);
  float* sdec_d = upload(s_dec, (size_t)B * 128);
  uint64_t* seeds_d = seeds ? upload(seeds, B) : nullptr;
  float* noise_d = nullptr;
  long long* noise_off_d = nullptr;
  if (noise) {
    std::vector<long long> off(B);
    long long t = 0;
    for (int b = 0; b < B; b++) off[b] = t, t += 600LL * 9 * items_h[b].n;
    noise_d = upload(noise, (size_t)t);
    noise_off_d = upload(off.data(), B);
  }
  times_compute_begin();
  cur_B = B;
  float* xcat0 = ar.get<float>((size_t)LN * X0_LD);
  float* f0 = ar.get<float>((size_t)2 * LN);
  float* nc = ar.get<float>((size_t)2 * LN);
  check(launch_gather_rows(asr_d, 512, tab1_d, LN, 512, xcat0, X0_LD, st), "gather_rows");
  check(launch_gather_rows(f0c_d, 1, tab2_d, 2 * LN, 1, f0, 1, st), "gather_rows");
  check(launch_gather_rows(nc_d, 1, tab2_d, 2 * LN, 1, nc, 1, st), "gather_rows");
  const int wdec = m.fc_dec.cout;
  float* gb_dec = ar.get<float>((size_t)B * wdec);
  linear(m.fc_dec, sdec_d, 128, B, gb_dec, wdec);
  float* audio = decode_core(B, items_h, items_d, col_item_d, LN, xcat0, f0, nc, gb_dec, wdec, seeds_d, noise_d,
                             noise_off_d);
  finish_audio(audio, LN, items_h, col_item_d, false);
  if (audio_out && !keep_audio_dev) {
    std::vector<void*> dst(B);
    std::vector<const void*> src(B);
    std::vector<size_t> nb(B);
    long long o = 0;
    for (int b = 0; b < B; b++) {
      dst[b] = audio_out + o, src[b] = audio_host + out_off[b], nb[b] = sizeof(float) * out_len[b];
      o += out_len[b];
    }
    parallel_copy(B, dst.data(), src.data(), nb.data());
  }
}

// ------------------------------------------------------------------------------ no-allocation decode

// Scratch of kk_decode_batch_noalloc: one static device array per GPU that loads this library
// (held until the process exits). Every call on a device shares it.
constexpr size_t NOALLOC_SCRATCH_BYTES = size_t(64) << 20;
constexpr int NOALLOC_MAX_ITEMS = 8;
constexpr int NOALLOC_MAX_FRAMES = 120;  // N-domain frames of a call, 2 gap frames per item included
static __device__ __align__(256) unsigned char g_noalloc_scratch[NOALLOC_SCRATCH_BYTES];

// Device address of g_noalloc_scratch on device `dev` (which must be current), looked up once per
// device under a std::once_flag, so threads driving engines on one device cannot race on the cache
// (a failed lookup throws and is retried by the next call). The host-side symbol is only a stand-in
// and must never be handed to a kernel. The cached address belongs to the device's primary context:
// a host application that resets the device (cudaDeviceReset) must not call this entry point again
// in the same process.
static void* noalloc_scratch(int dev) {
  static std::once_flag once[64];
  static void* addr[64] = {};
  if (dev < 0 || dev >= 64) throw KKError(KK_ERR_INVALID_ARG, "device ordinal above 63");
  std::call_once(once[dev], [dev] {
    void* p = nullptr;
    cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess) {
      cudaGetLastError();
      throw KKError(KK_ERR_CUDA, std::string("cudaGetSymbolAddress: ") + cudaGetErrorString(e));
    }
    addr[dev] = p;
  });
  return addr[dev];
}

void Engine::decode_noalloc(int B, const int32_t* n_frames, const float* asr, const float* f0_in, const float* n_in,
                            const float* s_dec, const uint64_t* seeds, const float* noise, float* audio_out) {
  KK_REQUIRE(B > 0, "empty batch");
  KK_REQUIRE(B <= NOALLOC_MAX_ITEMS, "kk_decode_batch_noalloc: more than 8 items in one call");
  KK_REQUIRE(n_frames && asr && f0_in && n_in && s_dec && audio_out, "null input or output pointer");
  ItemTab items_a[NOALLOC_MAX_ITEMS];
  int LN = 0, max_n = 0;
  long long tot = 0;
  for (int b = 0; b < B; b++) {
    KK_REQUIRE(n_frames[b] >= 1, "frame count out of range");
    KK_REQUIRE(n_frames[b] <= NOALLOC_MAX_FRAMES - GAP_N && LN + n_frames[b] + GAP_N <= NOALLOC_MAX_FRAMES,
               "kk_decode_batch_noalloc: more than 120 frames in one call (2 gap frames per item included)");
    items_a[b] = {0, 0, LN, n_frames[b]};
    LN += n_frames[b] + GAP_N;
    tot += n_frames[b];
    max_n = std::max(max_n, n_frames[b]);
  }
  LN = std::max(LN, MIN_LAYOUT_ROWS);  // as kk_decode_batch lays out the same call
  last_tokens = 0;
  last_frames = tot;
  KK_CUDA(cudaSetDevice(dev));
  struct Guard {  // leave the engine's normal (allocating) mode however the call ends
    Engine* e;
    ~Guard() {
      e->ar.clear_external();
      e->noalloc_active = false;
    }
  } guard{this};
  ar.set_external(noalloc_scratch(dev), NOALLOC_SCRATCH_BYTES);
  ar.set_poison(gap_canary ? st : nullptr);
  noalloc_active = true;
  KK_CUDA(cudaMemsetAsync(err_flag, 0, sizeof(int), st));
  int col_item[NOALLOC_MAX_FRAMES], tab1[NOALLOC_MAX_FRAMES], tab2[2 * NOALLOC_MAX_FRAMES];
  for (int i = 0; i < LN; i++) col_item[i] = tab1[i] = -1;
  for (int i = 0; i < 2 * LN; i++) tab2[i] = -1;
  long long r = 0;
  for (int b = 0; b < B; b++) {
    for (int i = 0; i < items_a[b].n; i++) {
      col_item[items_a[b].a + i] = b;
      tab1[items_a[b].a + i] = (int)(r + i);
    }
    for (int i = 0; i < 2 * items_a[b].n; i++) tab2[2 * items_a[b].a + i] = (int)(2 * r + i);
    r += items_a[b].n;
  }
  // synchronous copies straight from the caller's (pageable) buffers: no pinned staging
  auto put = [&](const void* h, size_t bytes) -> void* {
    void* d = ar.alloc(bytes);
    if (bytes) KK_CUDA(cudaMemcpyAsync(d, h, bytes, cudaMemcpyHostToDevice, st));
    return d;
  };
  long long noise_off[NOALLOC_MAX_ITEMS];
  long long nz = 0;
  for (int b = 0; b < B; b++) noise_off[b] = nz, nz += 600LL * 9 * items_a[b].n;
  ItemTab* items_d = (ItemTab*)put(items_a, sizeof(ItemTab) * B);
  int* col_item_d = (int*)put(col_item, sizeof(int) * LN);
  int* tab1_d = (int*)put(tab1, sizeof(int) * LN);
  int* tab2_d = (int*)put(tab2, sizeof(int) * 2 * LN);
  float* asr_d = (float*)put(asr, sizeof(float) * tot * 512);
  float* f0c_d = (float*)put(f0_in, sizeof(float) * 2 * tot);
  float* nc_d = (float*)put(n_in, sizeof(float) * 2 * tot);
  float* sdec_d = (float*)put(s_dec, sizeof(float) * B * 128);
  uint64_t* seeds_d = seeds ? (uint64_t*)put(seeds, sizeof(uint64_t) * B) : nullptr;
  float* noise_d = noise ? (float*)put(noise, sizeof(float) * nz) : nullptr;
  long long* noise_off_d = noise ? (long long*)put(noise_off, sizeof(long long) * B) : nullptr;
  cur_B = B;
  float* xcat0 = ar.get<float>((size_t)LN * X0_LD);
  float* f0 = ar.get<float>((size_t)2 * LN);
  float* nc = ar.get<float>((size_t)2 * LN);
  check(launch_gather_rows(asr_d, 512, tab1_d, LN, 512, xcat0, X0_LD, st), "gather_rows");
  check(launch_gather_rows(f0c_d, 1, tab2_d, 2 * LN, 1, f0, 1, st), "gather_rows");
  check(launch_gather_rows(nc_d, 1, tab2_d, 2 * LN, 1, nc, 1, st), "gather_rows");
  const int wdec = m.fc_dec.cout;
  float* gb_dec = ar.get<float>((size_t)B * wdec);
  linear(m.fc_dec, sdec_d, 128, B, gb_dec, wdec);
  float* audio = decode_core(B, max_n, items_d, col_item_d, LN, xcat0, f0, nc, gb_dec, wdec, seeds_d, noise_d,
                             noise_off_d);
  long long o = 0;
  for (int b = 0; b < B; b++) {
    KK_CUDA(cudaMemcpyAsync(audio_out + o, audio + 600LL * items_a[b].a, sizeof(float) * 600LL * items_a[b].n,
                            cudaMemcpyDeviceToHost, st));
    o += 600LL * items_a[b].n;
  }
  int errh = 0;
  KK_CUDA(cudaMemcpyAsync(&errh, err_flag, sizeof(int), cudaMemcpyDeviceToHost, st));
  KK_CUDA(cudaStreamSynchronize(st));
  if (errh) throw KKError(KK_ERR_TIMEOUT, wait_error(errh));
}

// Bounded-wait self-test: a kernel on the engine stream waits, through the pipelines' own bounded
// mbarrier wait, on a barrier that nothing arrives on, with a limit of limit_ns; the wait gives up,
// raises the engine's error flag and returns, and the flag is read back exactly as after a forward.
void Engine::wait_selftest(long long limit_ns) {
  KK_REQUIRE(limit_ns >= 1000 && limit_ns <= 100000000LL, "wait limit outside [1 us, 100 ms]");
  KK_CUDA(cudaSetDevice(dev));
  KK_CUDA(cudaMemsetAsync(err_flag, 0, sizeof(int), st));
  check(launch_wait_selftest(err_flag, (unsigned long long)limit_ns, st), "wait_selftest");
  int errh = 0;
  KK_CUDA(cudaMemcpyAsync(&errh, err_flag, sizeof(int), cudaMemcpyDeviceToHost, st));
  KK_CUDA(cudaStreamSynchronize(st));
  if (errh) throw KKError(KK_ERR_TIMEOUT, wait_error(errh));
  throw KKError(KK_ERR_CUDA, "wait self-test: the unarrived barrier wait did not expire");
}

}  // namespace kk

// ------------------------------------------------------------------------------ C ABI

struct kk_engine {
  std::unique_ptr<kk::Engine> e;
};

static thread_local std::string g_create_error;

template <class F>
static kk_status guarded(kk_engine* h, F&& f) {
  try {
    f();
    if (h) h->e->err.clear();
    return KK_OK;
  } catch (const kk::KKError& x) {
    if (h) h->e->err = x.what();
    else g_create_error = x.what();
    return (kk_status)x.status;
  } catch (const std::bad_alloc&) {
    if (h) h->e->err = "host allocation failed";
    else g_create_error = "host allocation failed";
    return KK_ERR_OOM;
  } catch (const std::exception& x) {
    if (h) h->e->err = x.what();
    else g_create_error = x.what();
    return KK_ERR_CUDA;
  }
}

extern "C" {

kk_status kk_create(const char* path, int cuda_ordinal, int precision, kk_engine** out) {
  if (!out || !path) {
    g_create_error = "null argument";
    return KK_ERR_INVALID_ARG;
  }
  *out = nullptr;
  if (precision != KK_PRECISION_FP32 && precision != KK_PRECISION_BF16) {
    g_create_error = "unknown precision";
    return KK_ERR_INVALID_ARG;
  }
  std::unique_ptr<kk_engine> h(new kk_engine{std::unique_ptr<kk::Engine>(new kk::Engine())});
  kk::Engine& e = *h->e;
  kk_status s = guarded(nullptr, [&] {
    int n = 0;
    KK_CUDA(cudaGetDeviceCount(&n));
    KK_REQUIRE(cuda_ordinal >= 0 && cuda_ordinal < n, "CUDA device ordinal out of range");
    cudaDeviceProp prop;
    KK_CUDA(cudaGetDeviceProperties(&prop, cuda_ordinal));
    if (prop.major != 10)
      throw kk::KKError(KK_ERR_CUDA, std::string("device ") + prop.name + " is not compute capability 10.x (sm_100a)");
    e.dev = cuda_ordinal;
    e.precision = precision;
    KK_CUDA(cudaSetDevice(cuda_ordinal));
    KK_CUDA(cudaStreamCreateWithFlags(&e.st, cudaStreamNonBlocking));
    KK_CUDA(cudaMalloc(&e.err_flag, sizeof(int)));
    e.wallocs.push_back(e.err_flag);
    KK_CUDA(cudaMemset(e.err_flag, 0, sizeof(int)));
    e.tc_ok = precision == KK_PRECISION_BF16 && kk::tc_available();
    kk::Checkpoint ck(path);
    e.load(ck);
    e.ident = std::string("cuda-b200 ") + (precision == KK_PRECISION_BF16 ? "bf16" : "fp32") +
              (e.tc_ok ? " tcgen05" : " simt");
  });
  if (s != KK_OK) return s;
  *out = h.release();
  return KK_OK;
}

void kk_destroy(kk_engine* h) { delete h; }

const char* kk_last_error(const kk_engine* h) { return h ? h->e->err.c_str() : g_create_error.c_str(); }

const char* kk_identity(const kk_engine* h) { return h ? h->e->ident.c_str() : ""; }

kk_status kk_forward_batch(kk_engine* h, int n_items, const int64_t* ids, const int32_t* ids_len, const float* ref_s,
                           const float* speed, const uint64_t* seeds, const float* noise, const int64_t* forced_dur,
                           int64_t* dur_out, int64_t* n_samples_out) {
  if (!h) return KK_ERR_INVALID_ARG;
  return guarded(h, [&] {
    h->e->out_off.clear();
    h->e->out_len.clear();
    std::vector<const float*> nz;
    std::vector<int64_t> nl;
    if (noise) {
      // concatenated draws: each item's share follows from its forced durations
      KK_REQUIRE(forced_dur, "replayed noise in kk_forward_batch requires forced durations (kk_forward_batch_noise "
                             "takes per-item draws with predicted durations)");
      KK_REQUIRE(n_items > 0 && ids_len, "null input pointer");
      long long o = 0, off = 0;
      for (int b = 0; b < n_items; b++) {
        long long nf = 0;
        for (int i = 0; i < ids_len[b]; i++) nf += forced_dur[o + i];
        o += ids_len[b];
        nz.push_back(noise + off);
        nl.push_back(600LL * 9 * nf);
        off += 600LL * 9 * nf;
      }
    }
    h->e->forward(n_items, ids, ids_len, ref_s, speed, seeds, noise ? nz.data() : nullptr,
                  noise ? nl.data() : nullptr, nullptr, forced_dur, dur_out, n_samples_out);
  });
}

kk_status kk_forward_batch_noise(kk_engine* h, int n_items, const int64_t* ids, const int32_t* ids_len,
                                 const float* ref_s, const float* speed, const uint64_t* seeds,
                                 const float* const* noise, const int64_t* noise_len, const float* rand_ini,
                                 const int64_t* forced_dur, int64_t* dur_out, int64_t* n_samples_out) {
  if (!h) return KK_ERR_INVALID_ARG;
  return guarded(h, [&] {
    h->e->out_off.clear();
    h->e->out_len.clear();
    h->e->forward(n_items, ids, ids_len, ref_s, speed, seeds, noise, noise_len, rand_ini, forced_dur, dur_out,
                  n_samples_out);
  });
}

kk_status kk_wait_selftest(kk_engine* h, int64_t limit_ns) {
  if (!h) return KK_ERR_INVALID_ARG;
  return guarded(h, [&] { h->e->wait_selftest(limit_ns); });
}

kk_status kk_fetch_audio(kk_engine* h, int item, float* dst, int64_t cap) {
  if (!h) return KK_ERR_INVALID_ARG;
  return guarded(h, [&] {
    kk::Engine& e = *h->e;
    KK_REQUIRE(item >= 0 && item < (int)e.out_off.size(), "item index out of range (no forward result)");
    KK_REQUIRE(!e.keep_audio_dev, "audio was kept on the device (KK_OPT_KEEP_AUDIO_ON_DEVICE)");
    KK_REQUIRE(!e.pcm16_out, "the last forward produced PCM_16 (KK_OPT_OUTPUT_PCM16): use kk_fetch_audio_pcm16");
    KK_REQUIRE(dst && cap >= e.out_len[item], "destination too small");
    memcpy(dst, e.audio_host + e.out_off[item], sizeof(float) * e.out_len[item]);
  });
}

kk_status kk_fetch_audio_all(kk_engine* h, float* const* dst, const int64_t* cap) {
  if (!h) return KK_ERR_INVALID_ARG;
  return guarded(h, [&] {
    kk::Engine& e = *h->e;
    KK_REQUIRE(!e.out_off.empty(), "no forward result");
    KK_REQUIRE(!e.keep_audio_dev, "audio was kept on the device (KK_OPT_KEEP_AUDIO_ON_DEVICE)");
    KK_REQUIRE(!e.pcm16_out, "the last forward produced PCM_16 (KK_OPT_OUTPUT_PCM16): use kk_fetch_audio_pcm16");
    KK_REQUIRE(dst && cap, "null argument");
    const int B = (int)e.out_off.size();
    std::vector<void*> d(B);
    std::vector<const void*> s(B);
    std::vector<size_t> nb(B);
    for (int b = 0; b < B; b++) {
      KK_REQUIRE(dst[b] && cap[b] >= e.out_len[b], "destination too small");
      d[b] = dst[b], s[b] = e.audio_host + e.out_off[b], nb[b] = sizeof(float) * e.out_len[b];
    }
    kk::parallel_copy(B, d.data(), s.data(), nb.data());
  });
}

kk_status kk_fetch_audio_pcm16(kk_engine* h, int item, int16_t* dst, int64_t cap, int64_t* clipped) {
  if (!h) return KK_ERR_INVALID_ARG;
  return guarded(h, [&] {
    kk::Engine& e = *h->e;
    KK_REQUIRE(item >= 0 && item < (int)e.out_off.size(), "item index out of range (no forward result)");
    KK_REQUIRE(!e.keep_audio_dev, "audio was kept on the device (KK_OPT_KEEP_AUDIO_ON_DEVICE)");
    KK_REQUIRE(e.pcm16_out && e.audio_host16, "the last forward produced f32 audio: use kk_fetch_audio");
    KK_REQUIRE(dst && cap >= e.out_len[item], "destination too small");
    memcpy(dst, e.audio_host16 + e.out_off[item], sizeof(int16_t) * e.out_len[item]);
    if (clipped) *clipped = e.out_clipped[item];
  });
}

kk_status kk_decode_batch(kk_engine* h, int n_items, const int32_t* n_frames, const float* asr, const float* f0,
                          const float* n, const float* s_dec, const uint64_t* seeds, const float* noise,
                          float* audio_out) {
  if (!h) return KK_ERR_INVALID_ARG;
  return guarded(h, [&] { h->e->decode(n_items, n_frames, asr, f0, n, s_dec, seeds, noise, audio_out); });
}

kk_status kk_decode_batch_noalloc(kk_engine* h, int n_items, const int32_t* n_frames, const float* asr, const float* f0,
                                  const float* n, const float* s_dec, const uint64_t* seeds, const float* noise,
                                  float* audio_out) {
  if (!h) return KK_ERR_INVALID_ARG;
  return guarded(h, [&] { h->e->decode_noalloc(n_items, n_frames, asr, f0, n, s_dec, seeds, noise, audio_out); });
}

kk_status kk_set_option(kk_engine* h, int option, int64_t value) {
  if (!h) return KK_ERR_INVALID_ARG;
  return guarded(h, [&] {
    if (option == KK_OPT_KEEP_AUDIO_ON_DEVICE) h->e->keep_audio_dev = value != 0;
    else if (option == KK_OPT_SYNC_EACH_STAGE) h->e->sync_each = value != 0;
    else if (option == KK_OPT_PROFILE) h->e->profile = value != 0;
    else if (option == KK_OPT_OUTPUT_PCM16) h->e->pcm16_out = value != 0;
    else if (option == KK_OPT_GAP_CANARY) h->e->gap_canary = value != 0;
    else if (option == KK_OPT_ATTENTION_F32) h->e->attn_f32 = value != 0;
    else if (option == KK_OPT_NEGCTL_NOMASK) {
      if (value != 0 && h->e->precision != KK_PRECISION_FP32)
        throw kk::KKError(KK_ERR_INVALID_ARG, "the no-mask negative control exists on the FP32 path only");
      h->e->negctl_nomask = value != 0;
    } else throw kk::KKError(KK_ERR_INVALID_ARG, "unknown option");
  });
}

kk_status kk_last_times(kk_engine* h, double out[4]) {
  if (!h || !out) return KK_ERR_INVALID_ARG;
  for (int i = 0; i < 4; i++) out[i] = h->e->last_times[i];
  return KK_OK;
}

int kk_profile_entry(kk_engine* h, int i, char* name, int name_cap, int64_t* launches, double* ms, double* flops) {
  if (!h) return -1;
  kk::Engine& e = *h->e;
  const int n = (int)e.prof_names.size();
  if (i < 0) return n;
  if (i >= n) return -1;
  if (name && name_cap > 0) {
    strncpy(name, e.prof_names[i].c_str(), (size_t)name_cap - 1);
    name[name_cap - 1] = 0;
  }
  if (launches) *launches = e.prof_launches[i];
  if (ms) *ms = e.prof_ms[i];
  if (flops) *flops = e.prof_flops[i];
  return n;
}

int kk_profile_launch(kk_engine* h, int i, char* cls, int cls_cap, double* ms, double* flops, double* bytes) {
  if (!h) return -1;
  kk::Engine& e = *h->e;
  const int n = (int)e.prof_log.size();
  if (i < 0) return n;
  if (i >= n) return -1;
  const auto& r = e.prof_log[i];
  if (cls && cls_cap > 0) {
    strncpy(cls, e.prof_names[r.cls].c_str(), (size_t)cls_cap - 1);
    cls[cls_cap - 1] = 0;
  }
  if (ms) *ms = r.ms;
  if (flops) *flops = r.flops;
  if (bytes) *bytes = r.bytes;
  return n;
}

void kk_profile_reset(kk_engine* h) {
  if (!h) return;
  kk::Engine& e = *h->e;
  std::fill(e.prof_launches.begin(), e.prof_launches.end(), 0);
  std::fill(e.prof_ms.begin(), e.prof_ms.end(), 0.0);
  std::fill(e.prof_flops.begin(), e.prof_flops.end(), 0.0);
  e.prof_log.clear();
}

int64_t kk_device_bytes(const kk_engine* h) { return h ? (int64_t)(h->e->wbytes + h->e->ar.bytes()) : 0; }

kk_status kk_memory_stats(const kk_engine* h, int64_t out[5]) {
  if (!h || !out) return KK_ERR_INVALID_ARG;
  out[0] = (int64_t)h->e->wbytes;
  out[1] = (int64_t)h->e->ar.bytes();
  out[2] = (int64_t)h->e->ar.peak();
  out[3] = h->e->last_tokens;
  out[4] = h->e->last_frames;
  return KK_OK;
}

kk_status kk_device_memory(int cuda_ordinal, int64_t* free_bytes, int64_t* total_bytes) {
  if (!free_bytes || !total_bytes) return KK_ERR_INVALID_ARG;
  int prev = 0;
  if (cudaGetDevice(&prev) != cudaSuccess || cudaSetDevice(cuda_ordinal) != cudaSuccess) {
    cudaGetLastError();
    return KK_ERR_CUDA;
  }
  size_t f = 0, t = 0;
  const cudaError_t e = cudaMemGetInfo(&f, &t);
  cudaSetDevice(prev);
  if (e != cudaSuccess) {
    cudaGetLastError();
    return KK_ERR_CUDA;
  }
  *free_bytes = (int64_t)f;
  *total_bytes = (int64_t)t;
  return KK_OK;
}

int64_t kk_launch_count(const kk_engine* h) { return h ? h->e->launches : 0; }

}  // extern "C"
