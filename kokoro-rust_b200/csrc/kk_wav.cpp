// WAV output of the synthesized audio (src/wav.rs): the canonical 44-byte RIFF/WAVE header,
// PCM_16 / float32 encoding with libsndfile's PCM_16 rule (sample * 0x7FFF, rounded half to even,
// clamped, clipped samples counted), and in-order assembly of per-line WAV parts into one file
// with a SHA-256 check of every part and an atomic rename. SHA-256 follows FIPS 180-4.
#include <errno.h>
#include <math.h>
#include <stdint.h>
#include <stdio.h>
#include <string.h>
#include <sys/stat.h>
#include <unistd.h>

#include <string>
#include <vector>

#include "../../include/kokoro_b200.h"

namespace {

thread_local std::string g_wav_error;

kk_status wfail(kk_status s, const std::string& m) {
  g_wav_error = m;
  return s;
}

constexpr uint64_t MAX_DATA_BYTES = 0xFFFFFFFFull - 36;  // RIFF size field is 36 + data, 32 bits

// ---------------------------------------------------------------------------- SHA-256 (FIPS 180-4)
struct Sha256 {
  uint32_t h[8];
  uint8_t buf[64];
  uint64_t len = 0;  // bytes hashed
  size_t fill = 0;
  Sha256() {
    static const uint32_t h0[8] = {0x6a09e667u, 0xbb67ae85u, 0x3c6ef372u, 0xa54ff53au,
                                   0x510e527fu, 0x9b05688cu, 0x1f83d9abu, 0x5be0cd19u};
    memcpy(h, h0, sizeof(h));
  }
  static uint32_t rotr(uint32_t x, int n) { return (x >> n) | (x << (32 - n)); }
  void block(const uint8_t* p) {
    static const uint32_t k[64] = {
        0x428a2f98u, 0x71374491u, 0xb5c0fbcfu, 0xe9b5dba5u, 0x3956c25bu, 0x59f111f1u, 0x923f82a4u, 0xab1c5ed5u,
        0xd807aa98u, 0x12835b01u, 0x243185beu, 0x550c7dc3u, 0x72be5d74u, 0x80deb1feu, 0x9bdc06a7u, 0xc19bf174u,
        0xe49b69c1u, 0xefbe4786u, 0x0fc19dc6u, 0x240ca1ccu, 0x2de92c6fu, 0x4a7484aau, 0x5cb0a9dcu, 0x76f988dau,
        0x983e5152u, 0xa831c66du, 0xb00327c8u, 0xbf597fc7u, 0xc6e00bf3u, 0xd5a79147u, 0x06ca6351u, 0x14292967u,
        0x27b70a85u, 0x2e1b2138u, 0x4d2c6dfcu, 0x53380d13u, 0x650a7354u, 0x766a0abbu, 0x81c2c92eu, 0x92722c85u,
        0xa2bfe8a1u, 0xa81a664bu, 0xc24b8b70u, 0xc76c51a3u, 0xd192e819u, 0xd6990624u, 0xf40e3585u, 0x106aa070u,
        0x19a4c116u, 0x1e376c08u, 0x2748774cu, 0x34b0bcb5u, 0x391c0cb3u, 0x4ed8aa4au, 0x5b9cca4fu, 0x682e6ff3u,
        0x748f82eeu, 0x78a5636fu, 0x84c87814u, 0x8cc70208u, 0x90befffau, 0xa4506cebu, 0xbef9a3f7u, 0xc67178f2u};
    uint32_t w[64];
    for (int i = 0; i < 16; i++)
      w[i] = (uint32_t)p[4 * i] << 24 | (uint32_t)p[4 * i + 1] << 16 | (uint32_t)p[4 * i + 2] << 8 | p[4 * i + 3];
    for (int i = 16; i < 64; i++) {
      const uint32_t s0 = rotr(w[i - 15], 7) ^ rotr(w[i - 15], 18) ^ (w[i - 15] >> 3);
      const uint32_t s1 = rotr(w[i - 2], 17) ^ rotr(w[i - 2], 19) ^ (w[i - 2] >> 10);
      w[i] = w[i - 16] + s0 + w[i - 7] + s1;
    }
    uint32_t a = h[0], b = h[1], c = h[2], d = h[3], e = h[4], f = h[5], g = h[6], hh = h[7];
    for (int i = 0; i < 64; i++) {
      const uint32_t t1 = hh + (rotr(e, 6) ^ rotr(e, 11) ^ rotr(e, 25)) + ((e & f) ^ (~e & g)) + k[i] + w[i];
      const uint32_t t2 = (rotr(a, 2) ^ rotr(a, 13) ^ rotr(a, 22)) + ((a & b) ^ (a & c) ^ (b & c));
      hh = g, g = f, f = e, e = d + t1, d = c, c = b, b = a, a = t1 + t2;
    }
    h[0] += a, h[1] += b, h[2] += c, h[3] += d, h[4] += e, h[5] += f, h[6] += g, h[7] += hh;
  }
  void update(const uint8_t* p, size_t n) {
    len += n;
    while (n > 0) {
      const size_t take = n < 64 - fill ? n : 64 - fill;
      memcpy(buf + fill, p, take);
      fill += take, p += take, n -= take;
      if (fill == 64) block(buf), fill = 0;
    }
  }
  std::string hex() {
    const uint64_t bits = len * 8;
    const uint8_t pad = 0x80;
    update(&pad, 1);
    const uint8_t z = 0;
    while (fill != 56) update(&z, 1);
    uint8_t lb[8];
    for (int i = 0; i < 8; i++) lb[i] = (uint8_t)(bits >> (56 - 8 * i));
    update(lb, 8);
    static const char* dg = "0123456789abcdef";
    std::string s;
    for (int i = 0; i < 8; i++)
      for (int j = 28; j >= 0; j -= 4) s += dg[(h[i] >> j) & 15];
    return s;
  }
};

void put_le(uint8_t* p, uint64_t v, int n) {
  for (int i = 0; i < n; i++) p[i] = (uint8_t)(v >> (8 * i));
}

int bits_of(int fmt) { return fmt == KK_WAV_FLOAT32 ? 32 : 16; }

}  // namespace

extern "C" KK_API const char* kk_wav_error(void) { return g_wav_error.c_str(); }

extern "C" KK_API kk_status kk_wav_header(int fmt, uint32_t sample_rate, uint64_t data_bytes, uint8_t out[44]) {
  if ((fmt != KK_WAV_PCM16 && fmt != KK_WAV_FLOAT32) || !out) return wfail(KK_ERR_INVALID_ARG, "bad format");
  if (data_bytes > MAX_DATA_BYTES)
    return wfail(KK_ERR_INVALID_ARG, "the audio (" + std::to_string(data_bytes) +
                                         " bytes) exceeds the 4 GiB limit of a WAV file; split the input into "
                                         "smaller files");
  const int bits = bits_of(fmt);
  memcpy(out, "RIFF", 4);
  put_le(out + 4, 36 + data_bytes, 4);
  memcpy(out + 8, "WAVEfmt ", 8);
  put_le(out + 16, 16, 4);
  put_le(out + 20, fmt == KK_WAV_FLOAT32 ? 3 : 1, 2);
  put_le(out + 22, 1, 2);
  put_le(out + 24, sample_rate, 4);
  put_le(out + 28, (uint32_t)(sample_rate * (uint32_t)bits / 8), 4);
  put_le(out + 32, bits / 8, 2);
  put_le(out + 34, bits, 2);
  memcpy(out + 36, "data", 4);
  put_le(out + 40, data_bytes, 4);
  return KK_OK;
}

extern "C" KK_API kk_status kk_wav_encode(const float* audio, int64_t n, uint32_t sample_rate, int fmt, uint8_t* out,
                                          int64_t cap, int64_t* n_bytes, int64_t* clipped) {
  if (n < 0 || (n > 0 && !audio)) return wfail(KK_ERR_INVALID_ARG, "bad audio");
  const uint64_t data = (uint64_t)n * (bits_of(fmt) / 8);
  if (n_bytes) *n_bytes = (int64_t)(44 + data);
  if (!out) return KK_OK;  // size query
  if (cap < (int64_t)(44 + data)) return wfail(KK_ERR_INVALID_ARG, "output buffer too small");
  kk_status s = kk_wav_header(fmt, sample_rate, data, out);
  if (s != KK_OK) return s;
  int64_t clip = 0;
  uint8_t* p = out + 44;
  if (fmt == KK_WAV_PCM16) {
    for (int64_t i = 0; i < n; i++) {
      const float v = nearbyintf(audio[i] * 32767.0f);  // round half to even (default rounding mode)
      int16_t q;
      if (!(v >= -32768.0f && v <= 32767.0f)) {  // out of range or NaN: counted, clamped (NaN -> 0)
        clip++;
        q = v != v ? 0 : (v < 0 ? -32768 : 32767);
      } else {
        q = (int16_t)v;
      }
      put_le(p + 2 * i, (uint16_t)q, 2);
    }
  } else {
    memcpy(p, audio, (size_t)n * 4);  // little-endian host
  }
  if (clipped) *clipped = clip;
  return KK_OK;
}

extern "C" KK_API kk_status kk_sha256_hex(const uint8_t* data, int64_t n, char out[65]) {
  if (n < 0 || (n > 0 && !data) || !out) return wfail(KK_ERR_INVALID_ARG, "bad arguments");
  Sha256 h;
  h.update(data, (size_t)n);
  const std::string s = h.hex();
  memcpy(out, s.c_str(), 65);
  return KK_OK;
}

// Data size of a WAV file written by kk_wav_encode, after checking its header (format, one channel,
// sample rate) and that the file size matches it (src/wav.rs:118-130).
static kk_status read_canonical(const char* path, int fmt, uint32_t rate, uint64_t* data) {
  FILE* f = fopen(path, "rb");
  if (!f) return wfail(KK_ERR_IO, std::string("opening ") + path + ": " + strerror(errno));
  uint8_t h[44];
  const size_t got = fread(h, 1, 44, f);
  fclose(f);
  if (got != 44) return wfail(KK_ERR_IO, std::string(path) + ": shorter than a WAV header");
  const uint64_t d = (uint64_t)h[40] | (uint64_t)h[41] << 8 | (uint64_t)h[42] << 16 | (uint64_t)h[43] << 24;
  uint8_t want[44];
  kk_status s = kk_wav_header(fmt, rate, d, want);
  if (s != KK_OK) return s;
  if (memcmp(h, want, 44) != 0)
    return wfail(KK_ERR_IO, std::string(path) + ": not a mono " + std::to_string(rate) + " Hz " +
                                (fmt == KK_WAV_FLOAT32 ? "Float32" : "Pcm16") + " WAV as written by kokoro");
  struct stat st;
  if (stat(path, &st) != 0) return wfail(KK_ERR_IO, std::string("stat ") + path);
  if ((uint64_t)st.st_size != 44 + d)
    return wfail(KK_ERR_IO, std::string(path) + ": size " + std::to_string((long long)st.st_size) +
                                " does not match its header (" + std::to_string(d) + " bytes of audio)");
  *data = d;
  return KK_OK;
}

extern "C" KK_API kk_status kk_wav_read_canonical(const char* path, int fmt, uint32_t sample_rate, uint64_t* data_bytes) {
  if (!path || !data_bytes) return wfail(KK_ERR_INVALID_ARG, "null argument");
  return read_canonical(path, fmt, sample_rate, data_bytes);
}

extern "C" KK_API kk_status kk_wav_assemble(int n_parts, const char* const* part_paths, const char* const* part_sha256,
                                            int fmt, uint32_t sample_rate, const char* dest, int sync,
                                            char sha256_out[65], uint64_t* data_bytes, uint64_t* samples) {
  if (n_parts < 0 || (n_parts > 0 && (!part_paths || !part_sha256)) || !dest)
    return wfail(KK_ERR_INVALID_ARG, "null argument");
  uint64_t total = 0;
  for (int i = 0; i < n_parts; i++) {
    uint64_t d = 0;
    kk_status s = read_canonical(part_paths[i], fmt, sample_rate, &d);
    if (s != KK_OK) return s;
    total += d;
  }
  uint8_t head[44];
  kk_status s = kk_wav_header(fmt, sample_rate, total, head);
  if (s != KK_OK) return s;
  const std::string d = dest;
  const size_t slash = d.find_last_of('/');
  const std::string dir = slash == std::string::npos ? "" : d.substr(0, slash + 1);
  const std::string name = slash == std::string::npos ? d : d.substr(slash + 1);
  if (name.empty()) return wfail(KK_ERR_INVALID_ARG, "output path has no file name");
  const std::string tmp = dir + "." + name + ".partial";
  FILE* out = fopen(tmp.c_str(), "wb");
  if (!out) return wfail(KK_ERR_IO, "creating " + tmp + ": " + strerror(errno));
  auto abandon = [&](kk_status st, const std::string& msg) {
    fclose(out);
    unlink(tmp.c_str());
    return wfail(st, msg);
  };
  Sha256 whole;
  if (fwrite(head, 1, 44, out) != 44) return abandon(KK_ERR_IO, "writing " + tmp);
  whole.update(head, 44);
  std::vector<uint8_t> buf(1 << 20);
  for (int i = 0; i < n_parts; i++) {
    FILE* f = fopen(part_paths[i], "rb");
    if (!f) return abandon(KK_ERR_IO, std::string("opening ") + part_paths[i]);
    Sha256 part;
    uint8_t h[44];
    if (fread(h, 1, 44, f) != 44) {
      fclose(f);
      return abandon(KK_ERR_IO, std::string(part_paths[i]) + ": shorter than a WAV header");
    }
    part.update(h, 44);
    size_t n;
    while ((n = fread(buf.data(), 1, buf.size(), f)) > 0) {
      part.update(buf.data(), n);
      whole.update(buf.data(), n);
      if (fwrite(buf.data(), 1, n, out) != n) {
        fclose(f);
        return abandon(KK_ERR_IO, "writing " + tmp);
      }
    }
    fclose(f);
    const std::string got = part.hex();
    if (got != part_sha256[i])
      return abandon(KK_ERR_IO, std::string(part_paths[i]) + " changed since it was synthesized (sha256 " + got +
                                    ", expected " + part_sha256[i] + ")");
  }
  if (fflush(out) != 0) return abandon(KK_ERR_IO, "writing " + tmp);
  if (sync && fsync(fileno(out)) != 0) return abandon(KK_ERR_IO, "fsync " + tmp);
  fclose(out);
  if (rename(tmp.c_str(), dest) != 0) {
    unlink(tmp.c_str());
    return wfail(KK_ERR_IO, std::string("moving the finished WAV to ") + dest + ": " + strerror(errno));
  }
  const std::string hx = whole.hex();
  if (sha256_out) memcpy(sha256_out, hx.c_str(), 65);
  if (data_bytes) *data_bytes = total;
  if (samples) *samples = total / (bits_of(fmt) / 8);
  return KK_OK;
}
