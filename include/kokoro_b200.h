/*
 * kokoro_b200.h -- C ABI of the B200-native Kokoro-82M batched ragged forward.
 *
 * This boundary replaces the reference crate's GPU layer: the Rust side keeps `Engine`
 * (src/engine.rs) and binds these symbols in place of `Gpu::new` + `GpuKokoro::with_gpu`
 * (src/gpu.rs:81-105, :685-724) and `GpuKokoro::forward_batch` (src/gpu_batch.rs:179-421).
 * Plain pointers and sizes only; no C++ or CUDA types cross it.
 *
 * Conventions (mirroring the reference's contract, src/gpu_batch.rs:14-24, src/engine.rs:190-241):
 *  - Status codes instead of panics; kk_last_error() gives the message of the last failure.
 *  - An engine is bound to one CUDA device and one stream and is NOT thread-safe: use one
 *    handle per GPU per host thread (the reference runs one GPU thread, src/cli.rs:625).
 *  - Host buffers belong to the caller. Device memory comes from a per-engine arena that grows
 *    on demand and is reused across calls; an allocation failure returns KK_ERR_OOM so the
 *    caller's split-the-batch-in-half policy (src/engine.rs:229-234) still works.
 *  - Results are per item, in input order.
 */
#ifndef KOKORO_B200_H
#define KOKORO_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#if defined(__GNUC__)
#define KK_API __attribute__((visibility("default")))
#else
#define KK_API
#endif

typedef enum {
  KK_OK = 0,
  KK_ERR_INVALID_ARG = 1, /* bad shapes / ids / speed (src/gpu_batch.rs:183-187) */
  KK_ERR_OOM = 2,         /* device or pinned-host allocation failed */
  KK_ERR_CUDA = 3,        /* any other CUDA runtime error */
  KK_ERR_TIMEOUT = 4,     /* a bounded in-kernel wait (a tcgen05 pipeline, attention or LSTM recurrence
                             mbarrier) gave up; the message names the error-flag code */
  KK_ERR_IO = 5           /* weight file missing, unreadable or malformed */
} kk_status;

typedef enum {
  KK_PRECISION_FP32 = 0, /* fp32 everywhere (SIMT FFMA); the parity path */
  KK_PRECISION_BF16 = 1  /* bf16 tensor-core (tcgen05) convs and GEMMs, fp32 accumulation; the LSTM
                            recurrence on tensor cores at fp32-level accuracy */
} kk_precision;

typedef struct kk_engine kk_engine;

/* Model constants (src/model.rs:12-19, src/vocoder.rs:8-11). */
#define KK_STYLE_DIM 128
#define KK_REF_S_DIM 256
#define KK_MAX_DUR 50
#define KK_CONTEXT_LEN 512
#define KK_SAMPLE_RATE 24000
#define KK_SAMPLES_PER_FRAME 600
#define KK_HARMONICS 9

/*
 * kk_create -- load a safetensors checkpoint (the reference's layout: raw state-dict names,
 * weight_norm as weight_v/weight_g, AdaIN affine optional), or the PyTorch checkpoint itself when
 * the path ends in .pth (see kk_pth_open), onto CUDA device `cuda_ordinal`.
 * Replaces Gpu::new (src/gpu.rs:81) + Weights::load (src/weights.rs:14) +
 * Kokoro::from_weights (src/model.rs:122) + GpuKokoro::with_gpu (src/gpu.rs:685).
 */
KK_API kk_status kk_create(const char* safetensors_path, int cuda_ordinal, int precision, kk_engine** out);

/* Release every device and host resource of the engine. NULL is a no-op. */
KK_API void kk_destroy(kk_engine* e);

/* Message of the last failure on this engine (or of the last kk_create when e is NULL). */
KK_API const char* kk_last_error(const kk_engine* e);

/* Engine identity string (part of the reference's resume keys, src/engine.rs:109-111). */
KK_API const char* kk_identity(const kk_engine* e);

/*
 * kk_forward_batch -- the batched ragged forward (GpuKokoro::forward_batch,
 * src/gpu_batch.rs:179; BatchItem src/gpu_batch.rs:19-24).
 *
 *  ids, ids_len   token ids of all items concatenated, pads included; ids_len[i] in [2, 512]
 *  ref_s          [n_items][256] style vectors (128 decoder + 128 prosody)
 *  speed          [n_items], finite and > 0
 *  seeds          [n_items] counter-noise seeds (ItemNoise::Counter), NULL = all zero
 *  noise          NULL, or replayed sine-noise draws (ItemNoise::Fixed) for every item,
 *                 concatenated, 600 * 9 * N_b floats per item; requires forced_dur, because the
 *                 concatenated buffer carries no per-item lengths (kk_forward_batch_noise takes
 *                 per-item draws with predicted durations, as the reference does)
 *  forced_dur     NULL, or per-token durations (>= 0, each item's sum >= 1), laid out like ids;
 *                 replaces the predicted durations (vocoder comparison mode)
 *  dur_out        [sum ids_len] durations used (predicted or forced), like ids; may be NULL
 *  n_samples_out  [n_items] audio length of each item, 600 * sum(dur); may be NULL
 *
 * The audio stays in the engine until the next forward call: read it with kk_fetch_audio.
 */
KK_API kk_status kk_forward_batch(kk_engine* e, int n_items, const int64_t* ids, const int32_t* ids_len,
                           const float* ref_s, const float* speed, const uint64_t* seeds,
                           const float* noise, const int64_t* forced_dur, int64_t* dur_out,
                           int64_t* n_samples_out);

/*
 * kk_forward_batch_noise -- kk_forward_batch with the reference's per-item noise choice
 * (ItemNoise, src/gpu_batch.rs:14-17; its use at src/gpu_batch.rs:325-340): item i replays
 * noise[i] (ItemNoise::Fixed) when noise is not NULL and noise[i] is not NULL, else it draws the
 * counter stream of seeds[i] (ItemNoise::Counter), so one batch may mix both. A replayed item's
 * draw count noise_len[i] must equal 600 * 9 * N_i for the durations the call uses, predicted or
 * forced, else the call fails with KK_ERR_INVALID_ARG ("fixed noise size mismatch for item i")
 * after the durations are known, as the reference's check does. rand_ini ([n_items][9] or NULL) is
 * the Fixed variant's initial phase: it must be finite and is otherwise unused, because the
 * reference adds it to the rad curve at sample 0 only, and the linear x1/300 downsample of the
 * phase never reads sample 0 (its first source position is 149.5). Other arguments as
 * kk_forward_batch.
 */
KK_API kk_status kk_forward_batch_noise(kk_engine* e, int n_items, const int64_t* ids, const int32_t* ids_len,
                                        const float* ref_s, const float* speed, const uint64_t* seeds,
                                        const float* const* noise, const int64_t* noise_len, const float* rand_ini,
                                        const int64_t* forced_dur, int64_t* dur_out, int64_t* n_samples_out);

/* Copy item `item`'s audio of the last forward into `dst` (capacity `cap` floats). */
KK_API kk_status kk_fetch_audio(kk_engine* e, int item, float* dst, int64_t cap);

/*
 * Copy every item's audio of the last forward at once: item i into dst[i] (capacity cap[i] floats),
 * on several host threads (the reference's forward_batch returns owned per-item Vec<f32>,
 * src/gpu_batch.rs:408-420; filling fresh caller buffers is page-fault bound, so the copies of
 * different items run in parallel: up to 16 threads, fewer when the environment variable
 * KK_FETCH_THREADS, read once per process, says so). No counterpart in the reference.
 */
KK_API kk_status kk_fetch_audio_all(kk_engine* e, float* const* dst, const int64_t* cap);

/*
 * Item `item`'s audio of the last forward run with KK_OPT_OUTPUT_PCM16, as PCM_16 samples
 * (capacity `cap`), and how many of its samples were clipped. The conversion is the reference's WAV
 * rule (src/wav.rs:76-84), done on the GPU so half the bytes cross PCIe. No counterpart in the
 * reference (it converts on the CPU in wav::encode).
 */
KK_API kk_status kk_fetch_audio_pcm16(kk_engine* e, int item, int16_t* dst, int64_t cap, int64_t* clipped);

/*
 * WAV output (src/wav.rs): the canonical 44-byte RIFF/WAVE header, PCM_16 (sample * 0x7FFF rounded
 * half to even, clamped, clipped samples counted; NaN is stored as 0 and counted) or float32 mono.
 */
typedef enum { KK_WAV_PCM16 = 0, KK_WAV_FLOAT32 = 1 } kk_wav_format;
/* Header for data_bytes of audio (wav::header, src/wav.rs:44-61); KK_ERR_INVALID_ARG above the
   4 GiB RIFF limit (data_bytes > 2^32 - 37), never a wrapped size field. */
KK_API kk_status kk_wav_header(int fmt, uint32_t sample_rate, uint64_t data_bytes, uint8_t out[44]);
/* Header + samples into out (capacity cap bytes); n_bytes receives 44 + data size (out may be NULL
   to query it), clipped the clipped-sample count (wav::encode, src/wav.rs:63-87). */
KK_API kk_status kk_wav_encode(const float* audio, int64_t n, uint32_t sample_rate, int fmt, uint8_t* out,
                               int64_t cap, int64_t* n_bytes, int64_t* clipped);
/* Data size of a WAV file written by kk_wav_encode after checking its header and file size
   (wav::read_canonical, src/wav.rs:118-130). */
KK_API kk_status kk_wav_read_canonical(const char* path, int fmt, uint32_t sample_rate, uint64_t* data_bytes);
/*
 * wav::assemble (src/wav.rs:132-187): concatenate the samples of WAV parts (each with the sha256
 * it had when written) into one WAV at dest, in order: one header, then every part's samples. The
 * result is written to a temporary file next to dest and renamed into place only when every part
 * was readable, canonical and unchanged (sha256), so dest is the complete new file or untouched.
 * sha256_out (65 bytes, may be NULL) receives the whole file's hex digest.
 */
KK_API kk_status kk_wav_assemble(int n_parts, const char* const* part_paths, const char* const* part_sha256, int fmt,
                                 uint32_t sample_rate, const char* dest, int sync, char sha256_out[65],
                                 uint64_t* data_bytes, uint64_t* samples);
/* Lower-case hex SHA-256 of n bytes (65 bytes with the terminator). */
KK_API kk_status kk_sha256_hex(const uint8_t* data, int64_t n, char out[65]);
/* Message of the last WAV-function failure on this thread. */
KK_API const char* kk_wav_error(void);

/*
 * PyTorch zip checkpoints (src/torchpt.rs): kokoro-v1_0.pth, a dict of state dicts, read as flat
 * "submodule.param" f32 tensors (a leading "module." dropped), and voice packs voices/<name>.pt, one
 * [rows, 1, 256] tensor. Deliberately restricted like the reference: STORED zip entries only, a small
 * pickle opcode set that is interpreted and never executed, and only the globals
 * collections.OrderedDict, torch._utils._rebuild_tensor_v2 and torch.FloatStorage; anything else
 * fails with KK_ERR_IO and a message naming it. kk_create also accepts a .pth checkpoint directly.
 */
typedef struct kk_pth kk_pth;
typedef enum { KK_PTH_CHECKPOINT = 0, KK_PTH_VOICE = 1 } kk_pth_kind;
/* Load a checkpoint (load_kmodel_checkpoint, src/torchpt.rs:302-319) or a voice pack
   (load_voice_pack, :322-335) into host memory. */
KK_API kk_status kk_pth_open(const char* path, int kind, kk_pth** out);
/* Tensors held (1 for a voice pack), in name order. */
KK_API int kk_pth_count(const kk_pth* p);
KK_API const char* kk_pth_name(const kk_pth* p, int i);
/* Rank of tensor i (-1 if out of range); its first min(rank, cap) extents go to dims. */
KK_API int kk_pth_shape(const kk_pth* p, int i, int64_t* dims, int cap);
/* Contiguous row-major f32 data of tensor i, valid until kk_pth_close. */
KK_API const float* kk_pth_data(const kk_pth* p, int i);
KK_API void kk_pth_close(kk_pth* p);
/* Message of the last kk_pth_open failure on this thread. */
KK_API const char* kk_pth_error(void);

/*
 * kk_decode_batch -- decoder + iSTFTNet generator only (the reference's
 * `decoder(asr, F0, N, ref_s[:, :128])`, src/gpu_batch.rs:299-420) on a ragged batch.
 *
 *  n_frames   [n_items] N_b frames per item (>= 1)
 *  asr        [sum N_b][512] aligned text features, time-major, items concatenated
 *  f0, n      [sum 2 N_b] F0 and N curves
 *  s_dec      [n_items][128] decoder styles
 *  seeds      [n_items] counter-noise seeds, NULL = all zero; noise: NULL or replayed draws
 *  audio_out  [sum 600 N_b] samples, items concatenated; may be NULL (audio kept on device)
 */
KK_API kk_status kk_decode_batch(kk_engine* e, int n_items, const int32_t* n_frames, const float* asr,
                          const float* f0, const float* n, const float* s_dec,
                          const uint64_t* seeds, const float* noise, float* audio_out);

/*
 * kk_decode_batch_noalloc -- kk_decode_batch for callers that cannot allocate device memory.
 * No counterpart in the reference crate.
 *
 * Who needs it: a caller that vocodes short chunks from a latency-bound thread (a streaming
 * audio callback cannot wait on cudaMalloc, which may synchronise the whole device and take
 * milliseconds) and a caller that shares a GPU under a fixed memory budget (the engine's arena
 * would otherwise grow to fit a new batch shape). This entry point allocates nothing: no device
 * memory, no pinned host memory, no events. Its scratch is one static device array of 64 MiB that
 * every GPU loading this library holds until the process exits; inputs are copied from, and the
 * audio written straight to, the caller's host buffers (synchronously).
 *
 * Limits: at most 8 items and 120 N-frames per call, counting 2 gap frames per item (one item
 * of up to 118 frames, about 2.95 s of audio); larger calls return KK_ERR_INVALID_ARG before any
 * work. audio_out must hold sum(600 * N_b) floats. Arguments and results otherwise as
 * kk_decode_batch.
 *
 * The first call on a device looks up the array's device address (once per device, with that
 * device current); make that first call before any stream capture. The address is kept for the
 * life of the process and belongs to the device's primary context: a host application that resets
 * the device (cudaDeviceReset) must not call this entry point again in that process. All calls on a
 * device share the array and it keeps the last call's contents: calls whose GPU work overlaps (two
 * threads or two engines on one device) race on it and must be serialised by the caller.
 */
KK_API kk_status kk_decode_batch_noalloc(kk_engine* e, int n_items, const int32_t* n_frames, const float* asr,
                                         const float* f0, const float* n, const float* s_dec,
                                         const uint64_t* seeds, const float* noise, float* audio_out);

/* Options (benchmark / diagnostics). */
typedef enum {
  KK_OPT_KEEP_AUDIO_ON_DEVICE = 1, /* 1: forward leaves audio on the device (no D2H) */
  KK_OPT_SYNC_EACH_STAGE = 2,      /* 1: synchronise after each stage (error localisation) */
  KK_OPT_PROFILE = 3,              /* 1: time every convolution / LSTM / attention launch with
                                      CUDA events on the engine stream (see kk_profile_entry) */
  KK_OPT_OUTPUT_PCM16 = 4,         /* 1: forward converts the audio to PCM_16 on the device (the WAV
                                      rule of kk_wav_encode) and copies only int16 to the host; read
                                      it with kk_fetch_audio_pcm16 (kk_fetch_audio then refuses) */
  KK_OPT_GAP_CANARY = 5,           /* tests, 1: every device buffer the engine takes for a call is
                                      first filled with NaN, so any element (a gap row above all) that
                                      a kernel reads before writing it poisons the output; outputs
                                      must not change. No counterpart in the reference */
  KK_OPT_NEGCTL_NOMASK = 6,        /* tests, 1 (FP32 mode only): convolutions read the gap rows of
                                      their input as they are instead of as zeros, the negative control
                                      of the reference's KOKORO_BATCH_NEGCTL_NOMASK
                                      (src/gpu_batch.rs:62-66): batched outputs must then change */
  KK_OPT_ATTENTION_F32 = 7         /* diagnostics, 1: the BF16 mode runs ALBERT's attention with the fp32
                                      kernel (the reference's f32 attention, src/gpu.rs:199-230) instead
                                      of the tcgen05 one, to measure what the bf16 Q / K / V / P of the
                                      tensor-core attention change. No counterpart in the reference */
} kk_option;
KK_API kk_status kk_set_option(kk_engine* e, int option, int64_t value);

/*
 * Device-side timings of the last kk_forward_batch / kk_decode_batch, from CUDA events recorded
 * on the engine's stream: out[0] = total ms (first host-to-device copy .. last device-to-host
 * copy), out[1] = compute ms (first kernel .. last kernel), out[2] = host-to-device bytes,
 * out[3] = device-to-host bytes. No counterpart in the reference (its bench times whole calls).
 */
KK_API kk_status kk_last_times(kk_engine* e, double out[4]);

/*
 * Kernel-class profile accumulated while KK_OPT_PROFILE is 1. Entry i (0-based) gives the class
 * name, its launches, total device milliseconds and algorithmic FLOPs (2 * MACs of the layer's
 * mathematical definition; a transposed convolution counts its own taps, not the zero taps of its
 * polyphase form). Returns the number of classes, or -1 for a bad index / engine.
 */
KK_API int kk_profile_entry(kk_engine* e, int i, char* name, int name_cap, int64_t* launches, double* ms,
                            double* flops);
/*
 * Launch i (0-based) of the launches profiled since the last kk_profile_reset: its class, device
 * time (ms), algorithmic FLOPs and algorithmic bytes (each input row read once, each output row
 * written once, residual rows read once, weights once). i < 0 returns the number of launches.
 * No counterpart in the reference (diagnostics of this engine).
 */
KK_API int kk_profile_launch(kk_engine* e, int i, char* cls, int cls_cap, double* ms, double* flops,
                             double* bytes);
KK_API void kk_profile_reset(kk_engine* e);

/*
 * kk_conv_selftest -- diagnostics: one 1-D convolution through the bf16 tcgen05 kernel on host
 * buffers (allocates and frees its own device memory; synchronous). No counterpart in the
 * reference: it exists so the kernel can be tested on its own against an fp32 convolution.
 *
 *  x      [rows_in or ceil(rows_in / 2) with up2][ldx] f32 input rows
 *  w      [cout][cin][K] f32 (torch Conv1d layout); bias [cout] or NULL
 *  coef   [n_items][cin] (A, B) pairs, AdaIN folded to x * A + B (in_mode 2 and 3)
 *  alpha  [cin] Snake alpha (in_mode 3)
 *  sc     [rows_out][ldsc] shortcut rows (out_mode 2)
 *  y      [rows_out][ldy] in/out (read for out_mode 1); x, y and sc need 16-byte aligned rows
 *         (row strides a multiple of 4 floats); columns cout .. round_up(cout, 4) - 1 of y may be
 *         overwritten (the kernel writes whole 16-byte units)
 *  stat   NULL, or [n_items][cout][2] f64: per (item, channel) sum and sum of squares of y
 *  timing_iters, ms_per_iter   when timing_iters > 0: the launch (with its input transform on the
 *         pre route) is repeated that many times more
 *         on the same device buffers and the mean device time per launch (CUDA events on the
 *         launching stream) is written to *ms_per_iter; y and stat then hold the repeated result
 */
typedef struct kk_conv_case {
  int cin, cout, K, dil, pad;
  int rows_in;   /* input-domain rows (after the optional nearest x2 upsample) */
  int ldx;
  int up2;       /* 1: input-domain row t reads x row t / 2 */
  int in_mode;   /* 0 as is, 1 gap rows -> 0, 2 leaky(AdaIN), 3 Snake(AdaIN), 4 leaky + gap mask */
  float slope;
  int rows_out, ldy;
  int out_mode;  /* 0 y = acc + bias, 1 y += acc + bias, 2 y = (acc + bias + sc) * oscale, 3 gelu */
  float oscale;
  int ldsc;
  int n_items;
  const int* item_in;   /* [rows_in] item of each input-domain row, -1 = gap */
  const int* item_out;  /* [rows_out] item of each output row, -1 = gap */
  int pre;              /* 1: transform the input once into bf16 window planes, then run the conv on
                           them (the route of layers with more than 128 output channels) */
} kk_conv_case;
KK_API kk_status kk_conv_selftest(int cuda_ordinal, const kk_conv_case* c, const float* x, const float* w,
                                  const float* bias, const float* coef, const float* alpha, const float* sc,
                                  float* y, double* stat, int timing_iters, double* ms_per_iter);
/*
 * kk_attention_selftest -- diagnostics: the BF16 mode's tcgen05 multi-head attention (12 heads of
 * 64) on host buffers. qkv [sum T][2304] rows [q | k | v] of n_items items of tok_len[i] in
 * [1, 512] rows each, concatenated; ctx [sum T][768] receives softmax(Q K^T / 8) V per item and
 * head. No counterpart in the reference (kernel-level test of src/gpu_batch.rs:429-442's math).
 */
KK_API kk_status kk_attention_selftest(int cuda_ordinal, int n_items, const int32_t* tok_len, const float* qkv,
                                       float* ctx);
/*
 * kk_attention_selftest_bf16 -- the same attention over bf16 qkv rows (bit patterns, 2 bytes per
 * element), the form the BF16 mode's QKV projection writes. Rows rounded to bf16 to nearest even
 * give the same ctx as kk_attention_selftest on the f32 rows, bit for bit.
 */
KK_API kk_status kk_attention_selftest_bf16(int cuda_ordinal, int n_items, const int32_t* tok_len,
                                            const uint16_t* qkv, float* ctx);
/*
 * kk_lstm_selftest -- diagnostics: one bidirectional LSTM recurrence (hidden 256) over 1 to 32
 * items, on host buffers. tc = 0: the fp32 cluster kernel (the FP32 mode's); tc = 1: the BF16 mode's
 * tcgen05 recurrence (fp32-level accuracy from fp16 split operands; |whh| must stay below 2^15). gx [sum len][2048] gate inputs (W_ih x + b_ih;
 * direction d, gate g (i, f, g, o), unit j at column d*1024 + g*256 + j), whh [2][1024][256],
 * bhh [2][1024]; out [sum len][512] receives h (direction d, unit j at d*256 + j). No counterpart in
 * the reference (kernel-level test of kernels/kokoro.cu:400-450's recurrence).
 */
KK_API kk_status kk_lstm_selftest(int cuda_ordinal, int tc, int n_items, const int32_t* len, const float* gx,
                                  const float* whh, const float* bhh, float* out);
/*
 * kk_wait_selftest -- diagnostics of the failure path: one kernel on the engine's stream waits, with
 * the bounded mbarrier wait every tcgen05 pipeline uses but a limit of limit_ns (1 us .. 100 ms), on
 * a barrier that nothing arrives on. The wait gives up, sets the engine's error flag and returns; the
 * call then returns KK_ERR_TIMEOUT with the flag's message, exactly as a forward whose wait expired
 * would, and the engine stays usable. No trap, no fault. No counterpart in the reference.
 */
KK_API kk_status kk_wait_selftest(kk_engine* e, int64_t limit_ns);

/* Message of the last kk_conv_selftest / kk_attention_selftest / kk_lstm_selftest failure on this thread. */
KK_API const char* kk_conv_selftest_error(void);

/* Bytes of device memory the engine currently holds (weights + arena). */
KK_API int64_t kk_device_bytes(const kk_engine* e);

/*
 * Device memory of the engine and of its last call, for the free-VRAM batch budget the reference
 * describes for its scheduler (docs/design/BATCHING.md:44-47; its code uses a fixed phoneme budget,
 * src/engine.rs:148-161): out[0] = weight bytes, out[1] = arena bytes held (reused by the next
 * call), out[2] = peak arena bytes in use during the last call, out[3] = phoneme tokens of the
 * last kk_forward_batch (0 after a decode), out[4] = frames of the last call.
 */
KK_API kk_status kk_memory_stats(const kk_engine* e, int64_t out[5]);

/* Free and total device memory of a CUDA device (cudaMemGetInfo). */
KK_API kk_status kk_device_memory(int cuda_ordinal, int64_t* free_bytes, int64_t* total_bytes);

/* Number of kernel launches issued by the engine since creation (counted on the host). */
KK_API int64_t kk_launch_count(const kk_engine* e);

#ifdef __cplusplus
}
#endif
#endif /* KOKORO_B200_H */
