/*
 * splitzip_oracle.c -- CPU restatement of the UnchainKV "splitzip" bf16 KV codec.
 *
 * TEST INFRASTRUCTURE ONLY.  This file is the parity checker for the CUDA
 * library in unchainkv_b200/csrc and the timed CPU baseline of bench.py.  Only
 * tests/, __graft_entry__.smoke() and bench.py's CPU-baseline / reference arm
 * may load it; the product path never does.
 *
 * Algorithm source (reference repo, path:line):
 *   top16 encode   native/unchain_kv/kvq_splitzip_cuda.cu:146-208, 381-414
 *   top16 decode   native/unchain_kv/kvq_splitzip_cuda.cu:210-284, 416-463
 *   fixed6/fixed5  native/unchain_kv/kvq_splitzip_cuda.cu:20-144, 292-379
 *   gather         src/unchain_kv/vllm_connector.py:2827-2869 (index_select over dim 1)
 *   CPU decoder    src/unchain_kv/vllm_connector.py:176-220
 *   modes 0/1/2    src/unchain_kv/vllm_connector.py:3204-3366 (encoder, packing),
 *   and fixed5     5168-5278 (receiver)
 *
 * Canonical form.  The reference GPU encoder is nondeterministic in three
 * places: escape-entry order (atomicAdd slot, .cu:177), unused escape slots
 * (uninitialised), and the fixed6/fixed5 palette order (atomicCAS claim,
 * .cu:37-46).  This restatement fixes each:
 *   - escape entries in ascending position order, unused slots zero;
 *   - on overflow (escapes > capacity): mode 255, count = capacity, the
 *     entries are the first `capacity` escapes by position;
 *   - fixed palette = distinct high bytes in ascending order, unused palette
 *     bytes zero; on palette overflow only mode byte 255 and the palette (the
 *     `limit` smallest distinct high bytes) are defined.
 * Everything else (header, body, codes, sizes, decline rules, return values)
 * follows the reference exactly.
 *
 * Pinning: tests/test_oracle_golden.py checks this file against vectors that
 * tests/golden/make_golden.py produced by running the reference's own CPU
 * code (the pure-Python top16 decoder, the torch mode-3/4 receiver, the
 * table builder and the palette ranking rule) and the reference's hand-built
 * top16 known-answer payload (tests/test_vllm_connector.py:333-371).
 */
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

/* ------------------------------------------------------------------ sizes */

uint64_t orc_top16_capacity(uint64_t n) { return (n + 199) / 200; }

uint64_t orc_top16_encoded_bytes(uint64_t n) {
  return 5 + n + (n + 1) / 2 + 5 * orc_top16_capacity(n);
}

uint64_t orc_fixed_encoded_bytes(uint64_t n, int bits) {
  if (bits == 5) return 33 + n + ((n + 7) / 8) * 5;
  return 65 + n + ((n + 3) / 4) * 3;
}

/* ------------------------------------------------------------ word views */

/* A packed word index i in [0, n) maps to the paged cache exactly as
 * torch.index_select(kv_layer, 1, ids) followed by a flat view does
 * (vllm_connector.py:2866) and as Top16DstIndex computes (.cu:210-224):
 * plane = i / plane_words, block = (i % plane_words) / block_words,
 * within = i % block_words, address = plane*plane_stride +
 * id(block)*block_stride + within.  block_words == 0 means a flat buffer. */
typedef struct {
  uint64_t n, plane_words, block_words, plane_stride, block_stride, block_start;
  const int64_t* ids;
} orc_layout;

static inline uint64_t orc_addr(const orc_layout* l, uint64_t i) {
  if (!l->block_words) return i;
  uint64_t plane = i / l->plane_words;
  uint64_t rem = i % l->plane_words;
  uint64_t blk = rem / l->block_words;
  uint64_t within = rem % l->block_words;
  uint64_t b = l->ids ? (uint64_t)l->ids[blk] : l->block_start + blk;
  return plane * l->plane_stride + b * l->block_stride + within;
}

static orc_layout flat_layout(uint64_t n) {
  orc_layout l;
  memset(&l, 0, sizeof l);
  l.n = n;
  return l;
}

static orc_layout block_layout(uint64_t block_count, uint64_t block_words,
                               uint64_t plane_stride, uint64_t block_stride,
                               uint64_t block_start, const int64_t* ids) {
  orc_layout l;
  l.n = 2 * block_count * block_words;
  l.plane_words = block_count * block_words;
  l.block_words = block_words;
  l.plane_stride = plane_stride;
  l.block_stride = block_stride;
  l.block_start = block_start;
  l.ids = ids;
  return l;
}

/* ------------------------------------------------------------ top16 encode */

static inline void put_u32le(uint8_t* p, uint32_t v) {
  p[0] = (uint8_t)v;
  p[1] = (uint8_t)(v >> 8);
  p[2] = (uint8_t)(v >> 16);
  p[3] = (uint8_t)(v >> 24);
}

static inline uint32_t get_u32le(const uint8_t* p) {
  return (uint32_t)p[0] | ((uint32_t)p[1] << 8) | ((uint32_t)p[2] << 16) |
         ((uint32_t)p[3] << 24);
}

/* One word of the top16 transform (.cu:170-191): body byte keeps the 7
 * mantissa bits and the sign; the 8-bit exponent goes through the plane's
 * inverse map; code 255 means "escape", which stores code 0. */
static inline void top16_word(uint16_t w, uint64_t plane, const uint8_t* tables,
                              uint8_t* body_byte, unsigned* code, unsigned* exp,
                              int* escape) {
  unsigned e = (w >> 7) & 0xFF;
  unsigned c = tables[plane * 256 + e];
  *body_byte = (uint8_t)((w & 0x7F) | ((w >> 8) & 0x80));
  *exp = e;
  *escape = c == 255;
  *code = *escape ? 0 : (c & 0x0F);
}

static int64_t top16_encode_layout(const uint16_t* src, const orc_layout* l,
                                   uint8_t* dst, uint64_t capacity,
                                   const uint8_t* tables) {
  uint64_t n = l->n;
  if (!src || !dst || !tables || n == 0 || n > 0xFFFFFFFFull) return 0;
  uint64_t code_bytes = (n + 1) / 2;
  uint64_t cap = orc_top16_capacity(n);
  uint64_t encoded = 5 + n + code_bytes + cap * 5;
  uint64_t scratch_offset = (encoded + 3) & ~3ull;
  if (encoded >= n * 2 || scratch_offset + 8 > capacity) return 0;
  uint8_t* body = dst + 5;
  uint8_t* codes = body + n;
  uint8_t* entries = codes + code_bytes;
  memset(codes, 0, code_bytes);
  memset(entries, 0, cap * 5);
  uint64_t half = n / 2;
  uint64_t count = 0;
  for (uint64_t i = 0; i < n; ++i) {
    uint16_t w = src[orc_addr(l, i)];
    unsigned code, exp;
    int escape;
    top16_word(w, i >= half, tables, &body[i], &code, &exp, &escape);
    if (escape) {
      if (count < cap) {
        put_u32le(entries + count * 5, (uint32_t)i);
        entries[count * 5 + 4] = (uint8_t)exp;
      }
      ++count;
    }
    codes[i / 2] |= (uint8_t)(code << ((i & 1) * 4));
  }
  dst[0] = count > cap ? 255 : 5;
  put_u32le(dst + 1, (uint32_t)(count > cap ? cap : count));
  return (int64_t)encoded;
}

/* kvq_splitzip_bf16_encode_top16 (.cu:381-414). */
int64_t orc_encode_top16(const uint16_t* src, uint64_t n, uint8_t* dst,
                         uint64_t capacity, const uint8_t* tables) {
  orc_layout l = flat_layout(n);
  return top16_encode_layout(src, &l, dst, capacity, tables);
}

/* Fused gather + encode: identical bytes to index_select(kv_layer, 1, ids)
 * (vllm_connector.py:2866) followed by encode_top16.  block_ids may be NULL
 * (contiguous run starting at block_start). */
int64_t orc_encode_top16_blocks(const uint16_t* cache, uint64_t plane_stride,
                                uint64_t block_stride, uint64_t block_words,
                                const int64_t* block_ids, uint64_t block_start,
                                uint64_t block_count, uint8_t* dst,
                                uint64_t capacity, const uint8_t* tables) {
  if (block_count == 0 || block_words == 0) return 0;
  orc_layout l = block_layout(block_count, block_words, plane_stride,
                              block_stride, block_start, block_ids);
  return top16_encode_layout(cache, &l, dst, capacity, tables);
}

/* Escape statistics of a top16 attempt without writing a stream: the number
 * of words whose exponent has no code.  Used by the pipeline tests. */
uint64_t orc_top16_escape_count(const uint16_t* src, uint64_t n,
                                const uint8_t* tables) {
  uint64_t half = n / 2, count = 0;
  for (uint64_t i = 0; i < n; ++i) {
    unsigned e = (src[i] >> 7) & 0xFF;
    count += tables[(i >= half) * 256 + e] == 255;
  }
  return count;
}

/* ------------------------------------------------------------ top16 decode */

static int64_t top16_decode_layout(const uint8_t* src, uint64_t encoded_bytes,
                                   uint16_t* dst, const orc_layout* l,
                                   const uint8_t* tables) {
  uint64_t n = l->n;
  uint64_t cap = orc_top16_capacity(n);
  if (encoded_bytes != 5 + n + (n + 1) / 2 + cap * 5) return 0;
  if (src[0] != 5) return (int64_t)(n * 2); /* .cu:235: writes nothing */
  const uint8_t* body = src + 5;
  const uint8_t* codes = body + n;
  const uint8_t* books = tables + 512;
  uint64_t half = n / 2;
  for (uint64_t i = 0; i < n; ++i) {
    unsigned code = (codes[i / 2] >> ((i & 1) * 4)) & 0x0F;
    unsigned exp = books[(i >= half) * 16 + code];
    uint8_t v = body[i];
    dst[orc_addr(l, i)] =
        (uint16_t)((v & 0x7F) | ((uint16_t)(v & 0x80) << 8) | (exp << 7));
  }
  /* ApplyTop16Escapes (.cu:253-284): slot < count && slot < capacity,
   * positions >= n skipped. */
  uint64_t count = get_u32le(src + 1);
  if (count > cap) count = cap;
  const uint8_t* entries = codes + (n + 1) / 2;
  for (uint64_t s = 0; s < count; ++s) {
    uint64_t pos = get_u32le(entries + s * 5);
    if (pos >= n) continue;
    uint16_t* w = &dst[orc_addr(l, pos)];
    *w = (uint16_t)((*w & 0x807F) | ((unsigned)entries[s * 5 + 4] << 7));
  }
  return (int64_t)(n * 2);
}

/* kvq_splitzip_bf16_decode_top16_blocks (.cu:416-451). */
int64_t orc_decode_top16_blocks(const uint8_t* src, uint64_t encoded_bytes,
                                uint16_t* dst, uint64_t count_words,
                                uint64_t block_count, uint64_t block_words,
                                uint64_t plane_stride, uint64_t block_stride,
                                uint64_t block_start, const int64_t* block_ids,
                                const uint8_t* tables) {
  if (!src || !dst || !tables || count_words == 0 || block_count == 0 ||
      block_words == 0 || count_words != 2 * block_count * block_words)
    return 0;
  orc_layout l = block_layout(block_count, block_words, plane_stride,
                              block_stride, block_start, block_ids);
  return top16_decode_layout(src, encoded_bytes, dst, &l, tables);
}

/* ------------------------------------------------------- fixed6 / fixed5 */

static int64_t fixed_encode_layout(const uint16_t* src, const orc_layout* l,
                                   uint8_t* dst, uint64_t capacity, int bits) {
  uint64_t n = l->n;
  if (!src || !dst || n == 0) return 0;
  if (bits != 5 && bits != 6) return 0;
  uint64_t encoded = orc_fixed_encoded_bytes(n, bits);
  uint64_t header = bits == 5 ? 33 : 65;
  uint64_t code_bytes = encoded - header - n;
  uint64_t scratch_offset = (encoded + 3) & ~3ull;
  if (encoded >= n * 2 || scratch_offset + 1032 > capacity) return 0;
  /* BuildPalette (.cu:28-49): the set of distinct high bytes. */
  uint8_t present[256];
  memset(present, 0, sizeof present);
  for (uint64_t i = 0; i < n; ++i) present[src[orc_addr(l, i)] >> 8] = 1;
  unsigned limit = bits == 5 ? 32 : 64;
  int rank[256];
  unsigned distinct = 0;
  memset(dst + 1, 0, limit);
  for (unsigned h = 0; h < 256; ++h) {
    rank[h] = -1;
    if (!present[h]) continue;
    if (distinct < limit) dst[1 + distinct] = (uint8_t)h;
    rank[h] = (int)distinct++;
  }
  if (distinct > limit) {
    dst[0] = 255; /* EncodeFixed6/5 overflow (.cu:59-62, 86-89) */
    return (int64_t)encoded;
  }
  dst[0] = bits == 5 ? 4 : 3;
  uint8_t* low = dst + header;
  uint8_t* codes = low + n;
  memset(codes, 0, code_bytes);
  for (uint64_t i = 0; i < n; ++i) {
    uint16_t w = src[orc_addr(l, i)];
    low[i] = (uint8_t)(w & 0xFF);
    unsigned code = (unsigned)rank[w >> 8];
    if (bits == 6) {
      /* 4 codes -> 3 bytes little endian (.cu:69-81). */
      uint64_t g = i / 4;
      uint32_t shift = (uint32_t)(i % 4) * 6;
      uint32_t v = (code & 0x3F) << shift;
      codes[g * 3] |= (uint8_t)v;
      codes[g * 3 + 1] |= (uint8_t)(v >> 8);
      codes[g * 3 + 2] |= (uint8_t)(v >> 16);
    } else {
      /* 8 codes -> 5 bytes little endian (.cu:96-110). */
      uint64_t g = i / 8;
      uint32_t shift = (uint32_t)(i % 8) * 5;
      uint64_t v = (uint64_t)(code & 0x1F) << shift;
      for (int b = 0; b < 5; ++b) codes[g * 5 + b] |= (uint8_t)(v >> (8 * b));
    }
  }
  return (int64_t)encoded;
}

/* kvq_splitzip_bf16_encode_mode (.cu:292-333). */
int64_t orc_encode_mode(const uint16_t* src, uint64_t n, uint8_t* dst,
                        uint64_t capacity, int bits) {
  orc_layout l = flat_layout(n);
  return fixed_encode_layout(src, &l, dst, capacity, bits);
}

int64_t orc_encode_mode_blocks(const uint16_t* cache, uint64_t plane_stride,
                               uint64_t block_stride, uint64_t block_words,
                               const int64_t* block_ids, uint64_t block_start,
                               uint64_t block_count, uint8_t* dst,
                               uint64_t capacity, int bits) {
  if (block_count == 0 || block_words == 0) return 0;
  orc_layout l = block_layout(block_count, block_words, plane_stride,
                              block_stride, block_start, block_ids);
  return fixed_encode_layout(cache, &l, dst, capacity, bits);
}

/* kvq_splitzip_bf16_decode_fixed6_blocks (.cu:344-368 / DecodeFixed6
 * .cu:113-144). */
int64_t orc_decode_fixed6_blocks(const uint8_t* src, uint64_t encoded_bytes,
                                 uint16_t* dst, uint64_t count_words,
                                 uint64_t block_count, uint64_t block_words,
                                 uint64_t plane_stride, uint64_t block_stride,
                                 uint64_t block_start,
                                 const int64_t* block_ids) {
  if (!src || !dst || count_words == 0 || block_count == 0 ||
      block_words == 0 || count_words != 2 * block_count * block_words)
    return 0;
  uint64_t n = count_words;
  if (encoded_bytes != 65 + n + ((n + 3) / 4) * 3) return 0;
  if (src[0] != 3) return (int64_t)(n * 2);
  orc_layout l = block_layout(block_count, block_words, plane_stride,
                              block_stride, block_start, block_ids);
  const uint8_t* palette = src + 1;
  const uint8_t* low = src + 65;
  const uint8_t* codes = low + n;
  for (uint64_t i = 0; i < n; ++i) {
    uint64_t g = i / 4;
    uint32_t packed = (uint32_t)codes[g * 3] | ((uint32_t)codes[g * 3 + 1] << 8) |
                      ((uint32_t)codes[g * 3 + 2] << 16);
    unsigned code = (packed >> ((i % 4) * 6)) & 0x3F;
    dst[orc_addr(&l, i)] = (uint16_t)(((uint16_t)palette[code] << 8) | low[i]);
  }
  return (int64_t)(n * 2);
}

/* ------------------------------------------------ multi-threaded baseline */

/* The same canonical top16 stream, produced by nthreads host threads: each
 * thread encodes a contiguous slice and keeps its escapes in a private list;
 * a serial prefix over the per-slice counts then places the entries.  Used
 * only as the timed CPU baseline. */
int64_t orc_encode_top16_blocks_mt(const uint16_t* cache, uint64_t plane_stride,
                                   uint64_t block_stride, uint64_t block_words,
                                   const int64_t* block_ids,
                                   uint64_t block_start, uint64_t block_count,
                                   uint8_t* dst, uint64_t capacity,
                                   const uint8_t* tables, int nthreads) {
  if (block_count == 0 || block_words == 0) return 0;
  orc_layout l = block_layout(block_count, block_words, plane_stride,
                              block_stride, block_start, block_ids);
  uint64_t n = l.n;
  if (!cache || !dst || !tables || n > 0xFFFFFFFFull) return 0;
  uint64_t code_bytes = (n + 1) / 2;
  uint64_t cap = orc_top16_capacity(n);
  uint64_t encoded = 5 + n + code_bytes + cap * 5;
  if (encoded >= n * 2 || ((encoded + 3) & ~3ull) + 8 > capacity) return 0;
  if (nthreads < 1) nthreads = 1;
  uint8_t* body = dst + 5;
  uint8_t* codes = body + n;
  uint8_t* entries = codes + code_bytes;
  uint64_t* counts = (uint64_t*)calloc((size_t)nthreads + 1, sizeof(uint64_t));
  uint32_t** lists = (uint32_t**)calloc((size_t)nthreads, sizeof(uint32_t*));
  uint64_t half = n / 2;
  /* slices start on even words so a code byte never spans two threads */
  uint64_t per = ((n / (uint64_t)nthreads) + 2) & ~1ull;
#pragma omp parallel num_threads(nthreads)
  {
    int t = 0;
#ifdef _OPENMP
    t = omp_get_thread_num();
#endif
    uint64_t lo = (uint64_t)t * per, hi = lo + per;
    if (lo > n) lo = n;
    if (hi > n) hi = n;
    uint64_t room = (hi - lo) < cap + 1 ? (hi - lo) : cap + 1;
    uint32_t* list = (uint32_t*)malloc((size_t)(room ? room : 1) * 2 * sizeof(uint32_t));
    uint64_t c = 0;
    for (uint64_t i = lo; i < hi; i += 2) {
      uint8_t packed = 0;
      for (uint64_t k = 0; k < 2 && i + k < hi; ++k) {
        uint64_t idx = i + k;
        uint16_t w = cache[orc_addr(&l, idx)];
        unsigned code, exp;
        int escape;
        top16_word(w, idx >= half, tables, &body[idx], &code, &exp, &escape);
        if (escape) {
          if (c < room) {
            list[2 * c] = (uint32_t)idx;
            list[2 * c + 1] = exp;
          }
          ++c;
        }
        packed |= (uint8_t)(code << (k * 4));
      }
      codes[i / 2] = packed;
    }
    counts[t + 1] = c;
    lists[t] = list;
  }
  for (int t = 0; t < nthreads; ++t) counts[t + 1] += counts[t];
  uint64_t total = counts[nthreads];
  memset(entries, 0, cap * 5);
#pragma omp parallel for num_threads(nthreads) schedule(static)
  for (int t = 0; t < nthreads; ++t) {
    uint64_t first = counts[t], mine = counts[t + 1] - counts[t];
    for (uint64_t k = 0; k < mine && first + k < cap; ++k) {
      put_u32le(entries + (first + k) * 5, lists[t][2 * k]);
      entries[(first + k) * 5 + 4] = (uint8_t)lists[t][2 * k + 1];
    }
  }
  for (int t = 0; t < nthreads; ++t) free(lists[t]);
  free(lists);
  free(counts);
  dst[0] = total > cap ? 255 : 5;
  put_u32le(dst + 1, (uint32_t)(total > cap ? cap : total));
  return (int64_t)encoded;
}

int64_t orc_encode_mode_blocks_mt(const uint16_t* cache, uint64_t plane_stride,
                                  uint64_t block_stride, uint64_t block_words,
                                  const int64_t* block_ids,
                                  uint64_t block_start, uint64_t block_count,
                                  uint8_t* dst, uint64_t capacity, int bits,
                                  int nthreads) {
  if (block_count == 0 || block_words == 0 || bits != 6) {
    return orc_encode_mode_blocks(cache, plane_stride, block_stride,
                                  block_words, block_ids, block_start,
                                  block_count, dst, capacity, bits);
  }
  orc_layout l = block_layout(block_count, block_words, plane_stride,
                              block_stride, block_start, block_ids);
  uint64_t n = l.n;
  if (!cache || !dst) return 0;
  uint64_t encoded = orc_fixed_encoded_bytes(n, 6);
  if (encoded >= n * 2 || ((encoded + 3) & ~3ull) + 1032 > capacity) return 0;
  if (nthreads < 1) nthreads = 1;
  uint8_t present[256];
  memset(present, 0, sizeof present);
#pragma omp parallel num_threads(nthreads)
  {
    uint8_t mine[256];
    memset(mine, 0, sizeof mine);
#pragma omp for schedule(static)
    for (int64_t i = 0; i < (int64_t)n; ++i) mine[cache[orc_addr(&l, (uint64_t)i)] >> 8] = 1;
#pragma omp critical
    for (int h = 0; h < 256; ++h) present[h] |= mine[h];
  }
  int rank[256];
  unsigned distinct = 0;
  memset(dst + 1, 0, 64);
  for (unsigned h = 0; h < 256; ++h) {
    rank[h] = -1;
    if (!present[h]) continue;
    if (distinct < 64) dst[1 + distinct] = (uint8_t)h;
    rank[h] = (int)distinct++;
  }
  if (distinct > 64) {
    dst[0] = 255;
    return (int64_t)encoded;
  }
  dst[0] = 3;
  uint8_t* low = dst + 65;
  uint8_t* codes = low + n;
  int64_t groups = (int64_t)((n + 3) / 4);
#pragma omp parallel for num_threads(nthreads) schedule(static)
  for (int64_t g = 0; g < groups; ++g) {
    uint32_t v = 0;
    for (uint64_t k = 0; k < 4; ++k) {
      uint64_t i = (uint64_t)g * 4 + k;
      if (i >= n) break;
      uint16_t w = cache[orc_addr(&l, i)];
      low[i] = (uint8_t)(w & 0xFF);
      v |= ((uint32_t)rank[w >> 8] & 0x3F) << (k * 6);
    }
    codes[g * 3] = (uint8_t)v;
    codes[g * 3 + 1] = (uint8_t)(v >> 8);
    codes[g * 3 + 2] = (uint8_t)(v >> 16);
  }
  return (int64_t)encoded;
}

int64_t orc_decode_fixed6_blocks_mt(const uint8_t* src, uint64_t encoded_bytes,
                                    uint16_t* dst, uint64_t count_words,
                                    uint64_t block_count, uint64_t block_words,
                                    uint64_t plane_stride,
                                    uint64_t block_stride, uint64_t block_start,
                                    const int64_t* block_ids, int nthreads) {
  if (!src || !dst || count_words == 0 || block_count == 0 ||
      block_words == 0 || count_words != 2 * block_count * block_words)
    return 0;
  uint64_t n = count_words;
  if (encoded_bytes != 65 + n + ((n + 3) / 4) * 3) return 0;
  if (src[0] != 3) return (int64_t)(n * 2);
  orc_layout l = block_layout(block_count, block_words, plane_stride,
                              block_stride, block_start, block_ids);
  const uint8_t* palette = src + 1;
  const uint8_t* low = src + 65;
  const uint8_t* codes = low + n;
  int64_t groups = (int64_t)((n + 3) / 4);
  if (nthreads < 1) nthreads = 1;
#pragma omp parallel for num_threads(nthreads) schedule(static)
  for (int64_t g = 0; g < groups; ++g) {
    uint32_t packed = (uint32_t)codes[g * 3] | ((uint32_t)codes[g * 3 + 1] << 8) |
                      ((uint32_t)codes[g * 3 + 2] << 16);
    for (uint64_t k = 0; k < 4; ++k) {
      uint64_t i = (uint64_t)g * 4 + k;
      if (i >= n) break;
      unsigned code = (packed >> (k * 6)) & 0x3F;
      dst[orc_addr(&l, i)] = (uint16_t)(((uint16_t)palette[code] << 8) | low[i]);
    }
  }
  return (int64_t)(n * 2);
}

int64_t orc_decode_top16_blocks_mt(const uint8_t* src, uint64_t encoded_bytes,
                                   uint16_t* dst, uint64_t count_words,
                                   uint64_t block_count, uint64_t block_words,
                                   uint64_t plane_stride, uint64_t block_stride,
                                   uint64_t block_start,
                                   const int64_t* block_ids,
                                   const uint8_t* tables, int nthreads) {
  if (!src || !dst || !tables || count_words == 0 || block_count == 0 ||
      block_words == 0 || count_words != 2 * block_count * block_words)
    return 0;
  uint64_t n = count_words;
  uint64_t cap = orc_top16_capacity(n);
  if (encoded_bytes != 5 + n + (n + 1) / 2 + cap * 5) return 0;
  if (src[0] != 5) return (int64_t)(n * 2);
  orc_layout l = block_layout(block_count, block_words, plane_stride,
                              block_stride, block_start, block_ids);
  const uint8_t* body = src + 5;
  const uint8_t* codes = body + n;
  const uint8_t* books = tables + 512;
  uint64_t half = n / 2;
  if (nthreads < 1) nthreads = 1;
#pragma omp parallel for num_threads(nthreads) schedule(static)
  for (int64_t s = 0; s < (int64_t)n; ++s) {
    uint64_t i = (uint64_t)s;
    unsigned code = (codes[i / 2] >> ((i & 1) * 4)) & 0x0F;
    unsigned exp = books[(i >= half) * 16 + code];
    uint8_t v = body[i];
    dst[orc_addr(&l, i)] =
        (uint16_t)((v & 0x7F) | ((uint16_t)(v & 0x80) << 8) | (exp << 7));
  }
  uint64_t count = get_u32le(src + 1);
  if (count > cap) count = cap;
  const uint8_t* entries = codes + (n + 1) / 2;
  for (uint64_t s = 0; s < count; ++s) {
    uint64_t pos = get_u32le(entries + s * 5);
    if (pos >= n) continue;
    uint16_t* w = &dst[orc_addr(&l, pos)];
    *w = (uint16_t)((*w & 0x807F) | ((unsigned)entries[s * 5 + 4] << 7));
  }
  return (int64_t)(n * 2);
}

int orc_max_threads(void) {
#ifdef _OPENMP
  return omp_get_max_threads();
#else
  return 1;
#endif
}

/* ------------------------------------------- receiver modes 0, 1, 2 and 4 */
/*
 * The reference's torch-op codec (the connector's path for tensors the CUDA
 * library does not take): encoder src/unchain_kv/vllm_connector.py:3204-3343,
 * bit packing :3345-3366, receiver :5168-5278.  Codes are packed LSB first:
 * code i of width w sits at bits [i*w, i*w + w) of the plane.
 *
 * The encoder tries, in order, and keeps the first form smaller than raw:
 *   mode 2, sign/magnitude, when the 7-bit magnitudes of the high bytes span
 *     fewer than 7 bits: [0]=2 [1]=width [2]=min magnitude, the n low bytes,
 *     n sign bits, n (magnitude - min) fields of `width` bits;
 *   mode 0, palette of the distinct high bytes, when it has at most 128
 *     entries: [0]=0 [1]=width=max(1, bitlen(distinct-1)) [2,258) the
 *     distinct high bytes ascending then zeros, the n low bytes, n codes;
 *   mode 1, nibble planes: [0]=1 [1,5) the widths of nibbles 0-3 (bits 0-3,
 *     4-7, 8-11, 12-15; 1 for <= 2 distinct values, 2 for <= 4, else 4),
 *     [5,69) four 16-byte palettes (distinct nibble values ascending, then
 *     zeros), then the four code planes.
 * Returns the stream length, or 0 when no form is smaller than raw.
 */
static inline uint32_t bitlen32(uint32_t v) {
  uint32_t b = 0;
  while (v) { ++b; v >>= 1; }
  return b;
}

static void put_bits(uint8_t* plane, uint64_t i, uint32_t width, uint32_t code) {
  const uint64_t bit = i * width;
  uint32_t v = code << (bit % 8);
  uint8_t* p = plane + bit / 8;
  for (uint32_t k = 0; k * 8 < (bit % 8) + width; ++k) p[k] |= (uint8_t)(v >> (8 * k));
}

static uint32_t get_bits(const uint8_t* plane, uint64_t i, uint32_t width) {
  const uint64_t bit = i * width;
  const uint8_t* p = plane + bit / 8;
  uint32_t v = 0;
  for (uint32_t k = 0; k * 8 < (bit % 8) + width; ++k) v |= (uint32_t)p[k] << (8 * k);
  return (v >> (bit % 8)) & ((1u << width) - 1u);
}

static int64_t torchop_encode_layout(const uint16_t* src, const orc_layout* l, uint8_t* dst,
                                     uint64_t capacity) {
  const uint64_t n = l->n, raw = 2 * n;
  uint32_t mag_min = 127, mag_max = 0;
  uint8_t seen[256] = {0};
  for (uint64_t i = 0; i < n; ++i) {
    const uint32_t high = src[orc_addr(l, i)] >> 8, mag = high & 0x7F;
    if (mag < mag_min) mag_min = mag;
    if (mag > mag_max) mag_max = mag;
    seen[high] = 1;
  }
  uint32_t width = bitlen32(mag_max - mag_min);
  if (width < 1) width = 1;
  if (width < 7) {
    const uint64_t sign_bytes = (n + 7) / 8, mag_bytes = (n * width + 7) / 8;
    const uint64_t encoded = 3 + n + sign_bytes + mag_bytes;
    if (encoded < raw) {
      if (encoded > capacity) return 0;
      memset(dst, 0, encoded);
      dst[0] = 2;
      dst[1] = (uint8_t)width;
      dst[2] = (uint8_t)mag_min;
      uint8_t* sign = dst + 3 + n;
      uint8_t* mags = sign + sign_bytes;
      for (uint64_t i = 0; i < n; ++i) {
        const uint16_t w = src[orc_addr(l, i)];
        dst[3 + i] = (uint8_t)(w & 0xFF);
        put_bits(sign, i, 1, w >> 15);
        put_bits(mags, i, width, ((w >> 8) & 0x7F) - mag_min);
      }
      return (int64_t)encoded;
    }
  }
  uint8_t rank[256];
  uint32_t distinct = 0;
  for (uint32_t h = 0; h < 256; ++h)
    if (seen[h]) rank[h] = (uint8_t)distinct++;
  width = bitlen32(distinct - 1);
  if (width < 1) width = 1;
  if (width < 8) {
    const uint64_t encoded = 258 + n + (n * width + 7) / 8;
    if (encoded < raw) {
      if (encoded > capacity) return 0;
      memset(dst, 0, encoded);
      dst[1] = (uint8_t)width;
      for (uint32_t h = 0; h < 256; ++h)
        if (seen[h]) dst[2 + rank[h]] = (uint8_t)h;
      uint8_t* codes = dst + 258 + n;
      for (uint64_t i = 0; i < n; ++i) {
        const uint16_t w = src[orc_addr(l, i)];
        dst[258 + i] = (uint8_t)(w & 0xFF);
        put_bits(codes, i, width, rank[w >> 8]);
      }
      return (int64_t)encoded;
    }
  }
  uint8_t nseen[4][16] = {{0}}, nrank[4][16];
  uint32_t nw[4], nsize[4];
  uint64_t encoded = 69;
  for (uint64_t i = 0; i < n; ++i) {
    const uint16_t w = src[orc_addr(l, i)];
    for (int p = 0; p < 4; ++p) nseen[p][(w >> (4 * p)) & 0xF] = 1;
  }
  for (int p = 0; p < 4; ++p) {
    uint32_t d = 0;
    for (uint32_t v = 0; v < 16; ++v)
      if (nseen[p][v]) nrank[p][v] = (uint8_t)d++;
    nw[p] = d <= 2 ? 1 : d <= 4 ? 2 : 4;
    nsize[p] = (uint32_t)((n * nw[p] + 7) / 8);
    encoded += nsize[p];
  }
  if (encoded >= raw || encoded > capacity) return 0;
  memset(dst, 0, encoded);
  dst[0] = 1;
  uint8_t* plane = dst + 69;
  for (int p = 0; p < 4; ++p) {
    dst[1 + p] = (uint8_t)nw[p];
    for (uint32_t v = 0; v < 16; ++v)
      if (nseen[p][v]) dst[5 + 16 * p + nrank[p][v]] = (uint8_t)v;
    for (uint64_t i = 0; i < n; ++i)
      put_bits(plane, i, nw[p], nrank[p][(src[orc_addr(l, i)] >> (4 * p)) & 0xF]);
    plane += nsize[p];
  }
  return (int64_t)encoded;
}

int64_t orc_encode_torchop_blocks(const uint16_t* cache, uint64_t plane_stride,
                                  uint64_t block_words, uint64_t block_stride,
                                  const int64_t* block_ids, uint64_t block_start,
                                  uint64_t block_count, uint8_t* dst,
                                  uint64_t capacity) {
  if (!cache || !dst || block_count == 0 || block_words == 0) return 0;
  orc_layout l = block_layout(block_count, block_words, plane_stride,
                              block_stride, block_start, block_ids);
  return torchop_encode_layout(cache, &l, dst, capacity);
}

/* Receiver decode of modes 0, 1, 2 and 4 (fixed5) into the paged cache,
 * with the receiver's checks (vllm_connector.py:5168-5278): a header field
 * out of range or a stream length other than the mode's declines (returns
 * 0); other modes decline too.  Returns 2n. */
int64_t orc_decode_modes_blocks(const uint8_t* src, uint64_t encoded_bytes,
                                uint16_t* dst, uint64_t block_count,
                                uint64_t block_words, uint64_t plane_stride,
                                uint64_t block_stride, uint64_t block_start,
                                const int64_t* block_ids) {
  if (!src || !dst || block_count == 0 || block_words == 0 || encoded_bytes == 0) return 0;
  orc_layout l = block_layout(block_count, block_words, plane_stride,
                              block_stride, block_start, block_ids);
  const uint64_t n = l.n;
  const uint8_t mode = src[0];
  if (mode == 0) {
    if (encoded_bytes < 258) return 0;
    const uint32_t width = src[1];
    if (width < 1 || width >= 8 || encoded_bytes != 258 + n + (n * width + 7) / 8) return 0;
    for (uint64_t i = 0; i < n; ++i)
      dst[orc_addr(&l, i)] =
          (uint16_t)((src[2 + get_bits(src + 258 + n, i, width)] << 8) | src[258 + i]);
  } else if (mode == 1) {
    if (encoded_bytes < 69) return 0;
    uint64_t total = 69;
    for (int p = 0; p < 4; ++p) {
      const uint32_t w = src[1 + p];
      if (w != 1 && w != 2 && w != 4) return 0;
      total += (n * w + 7) / 8;
    }
    if (encoded_bytes != total) return 0;
    for (uint64_t i = 0; i < n; ++i) {
      const uint8_t* plane = src + 69;
      uint32_t word = 0;
      for (int p = 0; p < 4; ++p) {
        const uint32_t w = src[1 + p];
        word |= (uint32_t)src[5 + 16 * p + get_bits(plane, i, w)] << (4 * p);
        plane += (n * w + 7) / 8;
      }
      dst[orc_addr(&l, i)] = (uint16_t)word;
    }
  } else if (mode == 2) {
    const uint32_t width = src[1], mag_min = src[2];
    if (width < 1 || width >= 7) return 0;
    const uint64_t sign_bytes = (n + 7) / 8;
    if (encoded_bytes != 3 + n + sign_bytes + (n * width + 7) / 8) return 0;
    for (uint64_t i = 0; i < n; ++i) {
      const uint32_t high = (get_bits(src + 3 + n, i, 1) << 7) |
                            (get_bits(src + 3 + n + sign_bytes, i, width) + mag_min);
      dst[orc_addr(&l, i)] = (uint16_t)((high << 8) | src[3 + i]);
    }
  } else if (mode == 4) {
    if (encoded_bytes != 33 + n + (n * 5 + 7) / 8) return 0;
    for (uint64_t i = 0; i < n; ++i)
      dst[orc_addr(&l, i)] =
          (uint16_t)((src[1 + get_bits(src + 33 + n, i, 5)] << 8) | src[33 + i]);
  } else {
    return 0;
  }
  return (int64_t)(2 * n);
}
