// KV snapshots in the reference's TNYKV001 format (cache_file.go:16-258):
//   "TNYKV001" | uint32 header length | JSON {"model_sha256":[32 bytes],
//   "float16":bool,"tokens":[ids]} | payload | SHA-256 of everything before.
// The payload holds the populated positions only, layer -> KV head -> keys,
// then values, each position's head_dim elements as little-endian float32 or
// raw binary16 bits (cachePayload, cache_file.go:203-228). Here the KV lives
// in pages of the device pool: k_kv_gather / k_kv_scatter move one layer
// between the pages and that file order.
#pragma once
#include <cstdint>
#include <cstring>
#include <string>
#include <vector>

#include "attention.cuh"

namespace tcu {

// SHA-256 (FIPS 180-4), streamed.
struct Sha256 {
  uint32_t h[8];
  uint8_t buf[64];
  uint64_t len = 0;
  size_t fill = 0;
  Sha256() {
    static const uint32_t init[8] = {0x6a09e667, 0xbb67ae85, 0x3c6ef372, 0xa54ff53a, 0x510e527f, 0x9b05688c, 0x1f83d9ab, 0x5be0cd19};
    memcpy(h, init, sizeof h);
  }
  static uint32_t rotr(uint32_t x, int n) { return (x >> n) | (x << (32 - n)); }
  void block(const uint8_t* p) {
    static const uint32_t k[64] = {
        0x428a2f98, 0x71374491, 0xb5c0fbcf, 0xe9b5dba5, 0x3956c25b, 0x59f111f1, 0x923f82a4, 0xab1c5ed5, 0xd807aa98, 0x12835b01,
        0x243185be, 0x550c7dc3, 0x72be5d74, 0x80deb1fe, 0x9bdc06a7, 0xc19bf174, 0xe49b69c1, 0xefbe4786, 0x0fc19dc6, 0x240ca1cc,
        0x2de92c6f, 0x4a7484aa, 0x5cb0a9dc, 0x76f988da, 0x983e5152, 0xa831c66d, 0xb00327c8, 0xbf597fc7, 0xc6e00bf3, 0xd5a79147,
        0x06ca6351, 0x14292967, 0x27b70a85, 0x2e1b2138, 0x4d2c6dfc, 0x53380d13, 0x650a7354, 0x766a0abb, 0x81c2c92e, 0x92722c85,
        0xa2bfe8a1, 0xa81a664b, 0xc24b8b70, 0xc76c51a3, 0xd192e819, 0xd6990624, 0xf40e3585, 0x106aa070, 0x19a4c116, 0x1e376c08,
        0x2748774c, 0x34b0bcb5, 0x391c0cb3, 0x4ed8aa4a, 0x5b9cca4f, 0x682e6ff3, 0x748f82ee, 0x78a5636f, 0x84c87814, 0x8cc70208,
        0x90befffa, 0xa4506ceb, 0xbef9a3f7, 0xc67178f2};
    uint32_t w[64];
    for (int i = 0; i < 16; i++) w[i] = (uint32_t)p[4 * i] << 24 | (uint32_t)p[4 * i + 1] << 16 | (uint32_t)p[4 * i + 2] << 8 | p[4 * i + 3];
    for (int i = 16; i < 64; i++) {
      const uint32_t s0 = rotr(w[i - 15], 7) ^ rotr(w[i - 15], 18) ^ (w[i - 15] >> 3);
      const uint32_t s1 = rotr(w[i - 2], 17) ^ rotr(w[i - 2], 19) ^ (w[i - 2] >> 10);
      w[i] = w[i - 16] + s0 + w[i - 7] + s1;
    }
    uint32_t a = h[0], b = h[1], c = h[2], d = h[3], e = h[4], f = h[5], g = h[6], hh = h[7];
    for (int i = 0; i < 64; i++) {
      const uint32_t t1 = hh + (rotr(e, 6) ^ rotr(e, 11) ^ rotr(e, 25)) + ((e & f) ^ (~e & g)) + k[i] + w[i];
      const uint32_t t2 = (rotr(a, 2) ^ rotr(a, 13) ^ rotr(a, 22)) + ((a & b) ^ (a & c) ^ (b & c));
      hh = g;
      g = f;
      f = e;
      e = d + t1;
      d = c;
      c = b;
      b = a;
      a = t1 + t2;
    }
    h[0] += a; h[1] += b; h[2] += c; h[3] += d; h[4] += e; h[5] += f; h[6] += g; h[7] += hh;
  }
  void update(const void* data, size_t n) {
    const uint8_t* p = (const uint8_t*)data;
    len += n;
    while (n > 0) {
      const size_t k = std::min(n, 64 - fill);
      memcpy(buf + fill, p, k);
      fill += k;
      p += k;
      n -= k;
      if (fill == 64) {
        block(buf);
        fill = 0;
      }
    }
  }
  void final(uint8_t out[32]) {
    const uint64_t bits = len * 8;
    const uint8_t one = 0x80, zero = 0;
    update(&one, 1);
    while (fill != 56) update(&zero, 1);
    uint8_t l[8];
    for (int i = 0; i < 8; i++) l[i] = (uint8_t)(bits >> (56 - 8 * i));
    update(l, 8);
    for (int i = 0; i < 8; i++)
      for (int j = 0; j < 4; j++) out[4 * i + j] = (uint8_t)(h[i] >> (24 - 8 * j));
  }
};

// One layer of a session's KV in file order: out[((g * 2 + kind) * T + t) *
// hd + e] (kind 0: keys, 1: values) from position t's page of the session's
// page table. Elements are copied as stored (float32 or binary16 bits).
__global__ void k_kv_gather(KVView kv, int layer, const int* page_table, int T, uint8_t* out) {
  const int es = kv.half ? 2 : 4;
  const size_t per = (size_t)T * kv.hd, total = (size_t)kv.kvh * 2 * per;
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < total; i += (size_t)gridDim.x * blockDim.x) {
    const int g = (int)(i / (2 * per)), kind = (int)(i / per % 2);
    const size_t r = i % per;
    const int t = (int)(r / kv.hd), e = (int)(r % kv.hd);
    const size_t o = kv.off(layer, page_table[t / kv.P], g, t % kv.P) + e;
    const uint8_t* src = (const uint8_t*)(kind ? kv.v : kv.k) + o * es;
    for (int b = 0; b < es; b++) out[i * es + b] = src[b];
  }
}

// The inverse of k_kv_gather: file-order elements of one layer into the pages.
__global__ void k_kv_scatter(KVView kv, int layer, const int* page_table, int T, const uint8_t* in) {
  const int es = kv.half ? 2 : 4;
  const size_t per = (size_t)T * kv.hd, total = (size_t)kv.kvh * 2 * per;
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < total; i += (size_t)gridDim.x * blockDim.x) {
    const int g = (int)(i / (2 * per)), kind = (int)(i / per % 2);
    const size_t r = i % per;
    const int t = (int)(r / kv.hd), e = (int)(r % kv.hd);
    const size_t o = kv.off(layer, page_table[t / kv.P], g, t % kv.P) + e;
    uint8_t* dst = (uint8_t*)(kind ? kv.v : kv.k) + o * es;
    for (int b = 0; b < es; b++) dst[b] = in[i * es + b];
  }
}

// The JSON header Go's encoding/json writes for cacheHeader
// (cache_file.go:18-22): a [32]byte is an array of numbers, nil tokens null.
inline std::string kv_header_json(const uint8_t model[32], bool half, const int32_t* tokens, int n) {
  std::string s = "{\"model_sha256\":[";
  for (int i = 0; i < 32; i++) s += (i ? "," : "") + std::to_string(model[i]);
  s += "],\"float16\":";
  s += half ? "true" : "false";
  s += ",\"tokens\":";
  if (n == 0) {
    s += "null";
  } else {
    s += "[";
    for (int i = 0; i < n; i++) s += (i ? "," : "") + std::to_string(tokens[i]);
    s += "]";
  }
  return s + "}";
}

// Reads that header back (whitespace and key order free, as encoding/json
// accepts them). Returns false on malformed input.
inline bool kv_header_parse(const std::string& js, uint8_t model[32], bool* half, std::vector<int32_t>* tokens) {
  size_t i = 0;
  auto ws = [&]() {
    while (i < js.size() && (js[i] == ' ' || js[i] == '\t' || js[i] == '\n' || js[i] == '\r')) i++;
  };
  auto lit = [&](const char* t) {
    ws();
    const size_t k = strlen(t);
    if (js.compare(i, k, t) != 0) return false;
    i += k;
    return true;
  };
  auto num = [&](long long* v) {
    ws();
    size_t j = i;
    if (j < js.size() && js[j] == '-') j++;
    const size_t d0 = j;
    while (j < js.size() && js[j] >= '0' && js[j] <= '9') j++;
    if (j == d0 || j - d0 > 18) return false;
    *v = std::stoll(js.substr(i, j - i));
    i = j;
    return true;
  };
  bool seen_model = false, seen_half = false;
  *half = false;
  tokens->clear();
  if (!lit("{")) return false;
  ws();
  if (lit("}")) return false;
  for (;;) {
    if (!lit("\"")) return false;
    const size_t e = js.find('"', i);
    if (e == std::string::npos) return false;
    const std::string key = js.substr(i, e - i);
    i = e + 1;
    if (!lit(":")) return false;
    if (key == "model_sha256") {
      if (!lit("[")) return false;
      for (int b = 0; b < 32; b++) {
        long long v;
        if ((b && !lit(",")) || !num(&v) || v < 0 || v > 255) return false;
        model[b] = (uint8_t)v;
      }
      if (!lit("]")) return false;
      seen_model = true;
    } else if (key == "float16") {
      if (lit("true"))
        *half = true;
      else if (!lit("false"))
        return false;
      seen_half = true;
    } else if (key == "tokens") {
      if (!lit("null")) {
        if (!lit("[")) return false;
        ws();
        if (!lit("]")) {
          for (;;) {
            long long v;
            if (!num(&v) || v < INT32_MIN || v > INT32_MAX) return false;
            tokens->push_back((int32_t)v);
            if (lit("]")) break;
            if (!lit(",")) return false;
          }
        }
      }
    } else {
      return false;
    }
    if (lit("}")) break;
    if (!lit(",")) return false;
  }
  ws();
  return i == js.size() && seen_model && seen_half;
}

}  // namespace tcu
