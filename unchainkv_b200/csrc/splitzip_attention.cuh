// Codec-aware GQA decode attention over splitzip streams (sm_100a).
//
// One decode query per request attends over that request's K/V of one layer,
// read straight from the request's transfer stream (the codec's output for
// the request's paged blocks, K plane then V plane) without decoding it into
// a paged cache first.  The reference receiver instead decodes the stream
// into its cache and runs attention on the bf16 copy.
//
// Shape (the Llama-3-8B decode of the benchmark configuration): 8 kv heads x
// 128 dims, 16-token blocks, GQA group g <= 8 q heads per kv head.
//
// Work: the blocks of all requests, in order, are split evenly over the
// persistent CTAs; an item is one CTA's run of blocks of one request (a CTA
// holds one or a few items).  Per item:
//   - producer warp: for each block, stages the K plane block (16 tokens x
//     8 heads x 128 dims), then the V plane block, into a ring of shared
//     memory stages by TMA (the rows' low bytes and 6-bit codes for fixed6,
//     their words for raw, their body bytes and 4-bit codes for top16);
//   - escape warp (top16 kernels only): from the stream's sorted escape
//     entries, writes into each top16 K stage's tail the escaped words'
//     share of S^T; AttnEscapeKernel adds the V escapes' share of O to the
//     items' partials;
//   - K warp h (kv head h): decodes its head's slice of each K block
//     straight into the A fragments of S^T = K Q^T (16 tokens x g q heads,
//     one m16n8k16 bf16 MMA per 16 dims) and hands the S^T fragments to the
//     V warp through a two-slot buffer with full/empty mbarriers;
//   - V warp h: keeps an online softmax per q head in fp32 (base 2), turns
//     P^T into the PV operand in registers (movmatrix), decodes its head's
//     slice of each V block straight into the A fragments of
//     O^T += V^T P^T (128 dims x g) and accumulates; P is split into two
//     bf16 parts (hi + lo) so that large V values do not amplify its
//     rounding;
//   - every item writes a partial (m, l, O) per q head to a workspace and
//     AttnCombineKernel merges them per request.
// Decoding into fragments needs no bf16 tile in shared memory: the MMAs'
// contraction and row orders are permuted so that each lane decodes
// consecutive dims of a few tokens (the permutation is applied to Q as well,
// and undone when O is written).  The tiles have g useful columns of 8
// (g = 4 for the benchmark), so they run on warp-level MMAs; the kernel is
// bound by the HBM read of the compressed K/V and by shared-memory traffic.
#pragma once

#include "splitzip_kernels.cuh"

namespace ukv {

constexpr int kAttnHeadDim = 128;
constexpr int kAttnBlockTokens = 16;
constexpr int kAttnKvHeads = kWarps;  // consumer warps of one plane
constexpr int kAttnConsumerWarps = 2 * kAttnKvHeads;  // a K and a V warp per kv head
constexpr int kAttnConsumers = 32 * kAttnConsumerWarps;
constexpr int kAttnThreads = kAttnConsumers + 32;     // + the producer warp
constexpr int kAttnKThreads = 32 * kAttnKvHeads;      // threads of the K warps
constexpr uint32_t kAttnBlockWords = kAttnBlockTokens * kAttnKvHeads * kAttnHeadDim;  // per plane
constexpr int kAttnStages = 6;  // K and V plane blocks alternate: 3 blocks in flight
// A stage holds one plane block as 16 token rows.  With kAttnRowPad = 16
// each row is copied to a slot 16 bytes longer than the row (consecutive
// rows start 4 banks apart, so fragment reads of 8 tokens at one offset do
// not collide) by one bulk copy per row; with 0 the rows are contiguous and
// a plane region goes by one bulk copy.
constexpr uint32_t kAttnRowPad = 0;
constexpr uint32_t kAttnRowWords = kAttnKvHeads * kAttnHeadDim;             // words of one token row
constexpr uint32_t kAttnLowPitch = kAttnRowWords + kAttnRowPad;             // fixed6 low bytes
constexpr uint32_t kAttnCodePitch = 3 * kAttnRowWords / 4 + kAttnRowPad;    // fixed6 codes
constexpr uint32_t kAttnRawPitch = 2 * kAttnRowWords + kAttnRowPad;         // raw words
constexpr uint32_t kAttnCodesOffset = kAttnBlockTokens * kAttnLowPitch + 16;  // fixed6 code rows inside a stage
constexpr uint32_t kAttnStageBytes = kAttnBlockTokens * kAttnRawPitch + 32;  // + room for the pads of whole regions
static_assert(kAttnCodesOffset + kAttnBlockTokens * kAttnCodePitch <= kAttnStageBytes, "fixed6 rows fit");
constexpr uint32_t kAttnSmemBytes = kAttnStages * kAttnStageBytes;  // dynamic shared memory: the ring
constexpr int kAttnMaxReqs = 64;
constexpr int kAttnMaxItems = 1024;
constexpr int kAttnMaxCtas = 320;
constexpr int kAttnMaxGroup = 8;
constexpr uint32_t kAttnRecord = kAttnHeadDim + 4;  // floats per (item, q head): o, m, l, 2 pad (16-byte records)

struct AttnReq {
  const uint8_t* stream;  // mode byte 3 (fixed6) or 6 (raw) stream of the request's blocks
  uint64_t stream_bytes;
  uint64_t n;             // words of the stream: 2 * blocks * kAttnBlockWords
  const uint16_t* q;      // bf16 [kv_heads * group][128]
  uint16_t* out;          // bf16 [kv_heads * group][128]
  const uint8_t* tables;  // the layer's 544-byte top16 table (books at 512, 528), or null
  uint32_t ctx;           // valid tokens (the last block may be partial)
  uint32_t first_item;
  uint32_t items;
  uint32_t pad;
};

struct AttnItem {
  uint32_t req;
  uint32_t block0;
  uint32_t blocks;
  uint32_t gblock0;  // the item's first block in the batch's order (all requests' blocks in turn)
};

template <int kMaxR, int kMaxI>
struct AttnBatch {
  uint32_t reqs;
  uint32_t items;
  uint32_t group;      // q heads per kv head
  float scale_log2;    // softmax scale * log2(e)
  float* partials;     // [items][kv_heads * group][kAttnRecord] (o, then m, l)
  float* scores;       // top16 batches: [batch blocks][kv heads][16 tokens][group] scaled scores, or null
  uint32_t ctas;
  uint16_t cta_item[kAttnMaxCtas + 1];  // items of CTA c: [cta_item[c], cta_item[c + 1])
  AttnReq req[kMaxR];
  AttnItem item[kMaxI];
};

struct AttnDesc {
  uint32_t item;   // or kEndTile
  uint32_t block;  // block of the request
  uint32_t plane;  // 0 = K, 1 = V
  uint32_t mode;
  uint32_t pad_x;
  uint32_t pad_y;
  uint32_t valid;  // valid tokens of the block
  uint32_t unused;
  uint32_t pad2[4];
  uint8_t pal[64];  // fixed6 palette of the request
};

using AttnRing = Ring<kAttnStages>;
using AttnPos = RingPos<kAttnStages>;

__device__ __forceinline__ uint32_t pack_bf16(float lo, float hi) {
  uint32_t r;
  asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
  return r;
}

__device__ __forceinline__ void mma_bf16(float (&c)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                         uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// Transpose an 8x8 bf16 matrix held in MMA fragment layout across the warp.
__device__ __forceinline__ uint32_t movmatrix_trans(uint32_t x) {
  uint32_t r;
  asm volatile("movmatrix.sync.aligned.m8n8.trans.b16 %0, %1;" : "=r"(r) : "r"(x));
  return r;
}

// Barrier of the attention kernel's K and V warps (named barrier 1).
__device__ __forceinline__ void attn_consumer_sync() {
  asm volatile("bar.sync 1, %0;" ::"n"(kAttnConsumers) : "memory");
}

// S^T hand-over from the K warp to the V warp of a head: two slots used in
// turn; full[slot] when written, empty[slot] when the V warp has read it.
// `valid` carries the block's valid tokens.
struct AttnHandoff {
  uint64_t full[2];
  uint64_t empty[2];
  uint32_t valid[2];
  uint32_t pad[2];
};

// The attention kernel's fixed6 pair table is stored swizzled: the entry of
// code pair idx = c0 | c1 << 6 (pal[c0] << 8 | pal[c1] << 24) sits at slot
// idx ^ (c1 & 31).  A warp's lookups then spread over the banks by c0 ^ c1
// rather than by c0 alone: neighbouring channels' codes concentrate on a few
// palette entries, and the decode shares the shared-memory pipe with the
// MMA operand reads.
__device__ __forceinline__ uint32_t pair_entry(const uint8_t* pal, uint32_t slot) {
  const uint32_t idx = slot ^ ((slot >> 6) & 31u);
  return (static_cast<uint32_t>(pal[idx & 63]) << 8) | (static_cast<uint32_t>(pal[idx >> 6]) << 24);
}

// Byte offset into the swizzled pair table of the code field f = 4 * idx.
__device__ __forceinline__ uint32_t pair_slot(uint32_t f) { return f ^ ((f >> 6) & 0x7Cu); }

// Pair-table lookup: the decoded bf16 word pair of the 12-bit code field at
// byte offset f (4 * field) with its two low bytes, which sit in bytes
// (sel & 1) * 2 and +1 of lw.
__device__ __forceinline__ uint32_t fixed6_pair(const uint8_t* pair, uint32_t f, uint32_t lw, bool upper) {
  return __byte_perm(lw, 0, upper ? 0x4342 : 0x4140) | *reinterpret_cast<const uint32_t*>(pair + pair_slot(f));
}

// Byte offset (4 * field) of 12-bit code field i (0..7) of 3 words.
__device__ __forceinline__ uint32_t fixed6_field(const uint32_t* c, int i) {
  switch (i) {
    case 0: return (c[0] << 2) & 0x3FFCu;
    case 1: return (c[0] >> 10) & 0x3FFCu;
    case 2: return __funnelshift_r(c[0], c[1], 22) & 0x3FFCu;
    case 3: return (c[1] >> 2) & 0x3FFCu;
    case 4: return (c[1] >> 14) & 0x3FFCu;
    case 5: return __funnelshift_r(c[1], c[2], 26) & 0x3FFCu;
    case 6: return (c[2] >> 6) & 0x3FFCu;
    default: return (c[2] >> 18) & 0x3FFCu;
  }
}

// One lane's share of staging a stage: `len` bytes at byte `off` of a stream
// of `glen` bytes, copied to a row slot from the 16-byte boundary at or
// below them (so the row starts `pad` bytes into the slot).  The 16-byte
// aligned middle goes by one bulk copy; the bytes before the stream's first
// or after its last 16-byte boundary by plain loads.
struct RowCopy {
  const uint8_t* first;  // the 16-byte boundary at or below the row
  const uint8_t* lo;     // bulk copy source, `bulk` bytes
  const uint8_t* row;    // the row, `len` bytes
  uint32_t bulk;
  uint32_t len;
  uint32_t pad;
};

__device__ __forceinline__ RowCopy plan_row_copy(const uint8_t* g, uint64_t glen, uint64_t off, uint32_t len) {
  const uintptr_t base = reinterpret_cast<uintptr_t>(g);
  const uintptr_t A = base + off, E = A + len;
  const uintptr_t F = A & ~static_cast<uintptr_t>(15);
  const uintptr_t gal = (base + 15) & ~static_cast<uintptr_t>(15);
  const uintptr_t gend = (base + glen) & ~static_cast<uintptr_t>(15);
  const uintptr_t lo = F > gal ? F : gal;
  const uintptr_t Eal = (E + 15) & ~static_cast<uintptr_t>(15);
  const uintptr_t hi = Eal < gend ? Eal : gend;
  RowCopy c;
  c.first = reinterpret_cast<const uint8_t*>(F);
  c.lo = reinterpret_cast<const uint8_t*>(lo);
  c.row = reinterpret_cast<const uint8_t*>(A);
  c.bulk = len > 0 && hi > lo ? static_cast<uint32_t>(hi - lo) : 0u;
  c.len = len;
  c.pad = static_cast<uint32_t>(A - F);
  return c;
}

// Issue the planned copy into the slot at `dst` (the barrier already
// expects the bulk bytes).
__device__ __forceinline__ void issue_row_copy(const RowCopy& c, uint8_t* dst, uint64_t* bar) {
  if (c.bulk > 0) bulk_g2s(dst + (c.lo - c.first), c.lo, c.bulk, bar);
  const uint8_t* end = c.row + c.len;
  const uint8_t* hi = c.bulk > 0 ? c.lo + c.bulk : c.row;
  for (const uint8_t* a = c.row; a < (c.bulk > 0 ? c.lo : c.row); ++a) dst[a - c.first] = *a;
  for (const uint8_t* a = hi > c.row ? hi : c.row; a < end; ++a) dst[a - c.first] = *a;
}

// Stage rows of token t: fixed6 low bytes, fixed6 codes, raw words.
__device__ __forceinline__ const uint8_t* low_row(const uint8_t* stage, uint32_t t) { return stage + t * kAttnLowPitch; }
__device__ __forceinline__ const uint8_t* code_row(const uint8_t* stage, uint32_t t) {
  return stage + kAttnCodesOffset + t * kAttnCodePitch;
}
__device__ __forceinline__ const uint8_t* raw_row(const uint8_t* stage, uint32_t t) { return stage + t * kAttnRawPitch; }

// The fixed6 inputs of NP word pairs of token t from word `dim` of the row:
// low bytes L (NP / 2 words) and codes C (3 NP / 8 words).
template <int NP>
__device__ __forceinline__ void fixed6_load(const AttnDesc& d, const uint8_t* stage, uint32_t t, uint32_t dim,
                                            uint32_t (&L)[NP / 2], uint32_t (&C)[3 * NP / 8]) {
  const uint8_t* low = low_row(stage, t) + dim;
  const uint8_t* codes = code_row(stage, t) + 3 * dim / 4;
  if ((d.pad_x | d.pad_y) == 0) {  // the stream's regions start on 16-byte boundaries
#pragma unroll
    for (int j = 0; j < NP / 8; ++j) {
      const uint4 l = reinterpret_cast<const uint4*>(low)[j];
      L[4 * j] = l.x; L[4 * j + 1] = l.y; L[4 * j + 2] = l.z; L[4 * j + 3] = l.w;
    }
    if constexpr (NP == 16) {  // 24 code bytes, 8-byte aligned
#pragma unroll
      for (int j = 0; j < 3; ++j) {
        const uint2 c = reinterpret_cast<const uint2*>(codes)[j];
        C[2 * j] = c.x;
        C[2 * j + 1] = c.y;
      }
    } else {  // 12 code bytes, 4-byte aligned
#pragma unroll
      for (int j = 0; j < 3 * NP / 8; ++j) C[j] = reinterpret_cast<const uint32_t*>(codes)[j];
    }
  } else {
    smem_read_words<NP / 2>(low, d.pad_x, L);
    smem_read_words<3 * NP / 8>(codes, d.pad_y, C);
  }
}

// Word pair i (words 2i, 2i + 1 from the loaded offset) of fixed6 inputs.
template <int NP>
__device__ __forceinline__ uint32_t fixed6_word_pair(const uint8_t* pair, const uint32_t (&L)[NP / 2],
                                                     const uint32_t (&C)[3 * NP / 8], int i) {
  return fixed6_pair(pair, fixed6_field(C + 3 * (i >> 3), i & 7), L[i >> 1], i & 1);
}

// Word pair i of token t from word `dim` of a raw row.
__device__ __forceinline__ uint32_t raw_word_pair(const AttnDesc& d, const uint8_t* stage, uint32_t t, uint32_t dim,
                                                  int i) {
  const uint8_t* row = raw_row(stage, t) + 2 * dim + 4 * i;
  if (d.pad_x == 0) return *reinterpret_cast<const uint32_t*>(row);
  uint32_t w[1];
  smem_read_words<1>(row, d.pad_x, w);
  return w[0];
}

// ---- top16 streams (the kTop16 kernel).  A stage holds the block plane's
// body rows (one byte a word) in place of the low-byte rows and its nibble
// rows (512 bytes a token) in place of the code rows.  The consumers decode
// every word from its book exponent, escaped words included; the escapes
// are corrected outside the MMAs:
//   - K stages: the escape warp writes into the stage's tail the escaped
//     words' share of S^T, (true - book value) x q summed per token and q
//     head, fp32 [token][kv head ^ (token & 7)][q head slot], 16 x 8 x 8;
//     the K warps add it to their S^T fragments;
//   - V stages: the V warps save their scaled scores, and AttnEscapeKernel
//     adds each escape's (true - book value) x p to the item's partial O.
constexpr uint32_t kAttnNibblePitch = kAttnRowWords / 2;
constexpr uint32_t kAttnEscCorr = 24640;
constexpr uint32_t kAttnCorrBytes = kAttnBlockTokens * kAttnKvHeads * kAttnMaxGroup * 4;
static_assert(kAttnCodesOffset + 16 + kAttnBlockTokens * kAttnNibblePitch <= kAttnEscCorr, "nibble rows");
static_assert(kAttnEscCorr % 16 == 0 && kAttnEscCorr + kAttnCorrBytes <= kAttnStageBytes, "escape share of S^T");

// Float index of (token t, kv head hk, q head slot q) in a K stage's escape
// share: the kv head is swizzled by the token, so the K warp's reads of 8
// tokens of one head fall on different banks.
__device__ __forceinline__ uint32_t corr_index(uint32_t t, uint32_t hk, uint32_t q) {
  return t * (kAttnKvHeads * kAttnMaxGroup) + ((hk ^ (t & 7u)) * kAttnMaxGroup) + q;
}

__device__ __forceinline__ const uint8_t* nibble_row(const uint8_t* stage, uint32_t t) {
  return stage + kAttnCodesOffset + t * kAttnNibblePitch;
}

// The top16 inputs of NP word pairs of token t from word `dim` of the row:
// body bytes B (NP / 2 words) and nibbles N (NP / 4 words).
template <int NP>
__device__ __forceinline__ void top16_load(const AttnDesc& d, const uint8_t* stage, uint32_t t, uint32_t dim,
                                           uint32_t (&B)[NP / 2], uint32_t (&N)[NP / 4]) {
  const uint8_t* body = low_row(stage, t) + dim;
  const uint8_t* nib = nibble_row(stage, t) + dim / 2;
  if ((d.pad_x | d.pad_y) == 0) {  // the stream's regions start on 16-byte boundaries
#pragma unroll
    for (int j = 0; j < NP / 8; ++j) {
      const uint4 v = reinterpret_cast<const uint4*>(body)[j];
      B[4 * j] = v.x; B[4 * j + 1] = v.y; B[4 * j + 2] = v.z; B[4 * j + 3] = v.w;
    }
    if constexpr (NP == 16) {  // 16 nibble bytes, 16-byte aligned
      const uint4 v = *reinterpret_cast<const uint4*>(nib);
      N[0] = v.x; N[1] = v.y; N[2] = v.z; N[3] = v.w;
    } else {  // 8 nibble bytes, 8-byte aligned
      const uint2 v = *reinterpret_cast<const uint2*>(nib);
      N[0] = v.x; N[1] = v.y;
    }
  } else {
    smem_read_words<NP / 2>(body, d.pad_x, B);
    smem_read_words<NP / 4>(nib, d.pad_y, N);
  }
}

// A top16 word pair: the body bytes of words 4q..4q+3 in bw (`upper` takes
// words 4q+2, 4q+3 instead of 4q, 4q+1) and the pair's code-byte table
// entry, which holds the two words' book exponents at bits 7 and 23.
__device__ __forceinline__ uint32_t top16_pair_t(uint32_t bw, uint32_t exps, bool upper) {
  return (__byte_perm(bw, 0, upper ? 0x3322 : 0x1100) & 0x807F807Fu) | exps;
}

// The bf16 value (as fp32) of a top16 word with body byte `body` (sign at
// bit 7, mantissa below) and exponent `e`.
__device__ __forceinline__ float top16_value(uint32_t body, uint32_t e) {
  return __uint_as_float((((body & 0x7Fu) | ((body & 0x80u) << 8)) | (e << 7)) << 16);
}

// First entry index in [0, total) whose position is >= target (total if
// none), entries sorted by position; warp-wide, 32 positions per round.
__device__ __forceinline__ uint32_t entries_lower_bound(const uint8_t* entries, uint32_t total, uint64_t target) {
  const uint32_t lane = threadIdx.x & 31;
  uint32_t lo = 0, hi = total;  // the answer lies in [lo, hi]
  for (int round = 0; round < 8 && hi - lo > 32; ++round) {
    const uint32_t step = (hi - lo + 31) / 32;
    const uint32_t idx = lo + (lane + 1) * step - 1;
    const bool below = idx < hi && entry_pos(entries, idx) < target;
    const uint32_t k = __popc(__ballot_sync(kFull, below));
    const uint32_t nlo = lo + k * step;
    hi = max(nlo, min(hi, lo + (k + 1) * step - 1));
    lo = nlo;
  }
  const uint32_t idx = lo + lane;
  const bool below = idx < hi && entry_pos(entries, idx) < target;
  return lo + __popc(__ballot_sync(kFull, below));
}

// 17 warps, one CTA per SM: a sub-partition hosting 5 of them allows 96
// registers per thread.
// kTop16: also reads top16 streams (mode 5), with the requests' tables.
template <int kMaxR, int kMaxI, bool kTop16>
__global__ void __launch_bounds__(kTop16 ? kAttnThreads + 32 : kAttnThreads, 1)
    AttnKernel(const __grid_constant__ AttnBatch<kMaxR, kMaxI> b) {
  extern __shared__ __align__(128) uint8_t ring[];
  __shared__ __align__(16) uint32_t pair[4096];
  __shared__ __align__(16) float4 scores[kAttnKvHeads][2][32];  // S^T fragments, two slots per head
  __shared__ __align__(16) AttnDesc D[kAttnStages];
  __shared__ AttnRing R;  // empty barriers count the kWarps == kAttnKvHeads warps of one plane
  __shared__ __align__(8) AttnHandoff hand[kAttnKvHeads];
  const int tid = threadIdx.x;
  const int lane = tid & 31;
  const int warp = tid >> 5;
  if (tid == 0) {
    for (int i = 0; i < kAttnStages; ++i) {
      // lane 0 of the producer, after the warp's copies are issued (and of
      // the escape warp, after the stage's escape tables)
      mbar_init(&R.full[i], kTop16 ? 2 : 1);
      mbar_init(&R.empty[i], kAttnKvHeads);
    }
  }
  if (tid < kAttnKvHeads) {
    for (int i = 0; i < 2; ++i) {
      mbar_init(&hand[tid].full[i], 1);
      mbar_init(&hand[tid].empty[i], 1);
    }
    fence_mbar_init();
  }
  __syncthreads();
  const uint32_t i_begin = blockIdx.x < b.ctas ? b.cta_item[blockIdx.x] : 0u;
  const uint32_t i_end = blockIdx.x < b.ctas ? b.cta_item[blockIdx.x + 1] : 0u;

  if (warp == kAttnConsumerWarps) {
    // ------------------------------------------------------------ producer
    // K then V of each block of each item of this CTA, one copy per token
    // row; the mode byte and the palette of the item's stream are read once
    // per item
    AttnPos p;
    for (uint32_t item = i_begin; item < i_end; ++item) {
      const AttnItem& I = b.item[item];
      const AttnReq& Q = b.req[I.req];
      uint32_t mode = __ldg(Q.stream);
      const uint64_t cap = (Q.n + 199) / 200;
      const uint64_t need = mode == 3 ? 65 + Q.n + 3 * ((Q.n + 3) / 4)
                            : mode == 6 ? 1 + 2 * Q.n
                            : (kTop16 && mode == 5 && Q.tables != nullptr) ? 5 + Q.n + (Q.n + 1) / 2 + 5 * cap
                                                                         : 0;
      if (need == 0 || need > Q.stream_bytes) {
        if (lane == 0) raise_error(nullptr);
        mode = 0;
      }
      const uint32_t pal = mode == 3 ? (static_cast<uint32_t>(__ldg(Q.stream + 1 + 2 * lane)) |
                                        (static_cast<uint32_t>(__ldg(Q.stream + 2 + 2 * lane)) << 8))
                                     : 0u;
      for (uint32_t k = 0; k < 2 * I.blocks; ++k) {
        const uint32_t blk = I.block0 + (k >> 1), plane = k & 1;
        producer_acquire(R, p, nullptr);
        AttnDesc& d = D[p.s];
        uint8_t* stage = ring + p.s * kAttnStageBytes;
        // lanes 0-15: the low-byte rows (fixed6) or the word rows (raw) of
        // tokens 0-15; lanes 16-31: the code rows (fixed6).  Rows are 1024
        // words apart, so every row has the same pad.
        // (with contiguous rows, lanes 0 and 16 copy the whole regions)
        const uint32_t t = lane & 15;
        const uint64_t wt = plane * (Q.n / 2) + (static_cast<uint64_t>(blk) * kAttnBlockTokens + t) * kAttnRowWords;
        constexpr uint32_t kRows = kAttnRowPad > 0 ? 1 : kAttnBlockTokens;  // rows per copy
        const bool copies = kAttnRowPad > 0 || t == 0;
        uint64_t off = 0;
        uint32_t len = 0;
        uint8_t* dst = stage;
        if (mode == 3 && copies) {
          off = lane < 16 ? 65 + wt : 65 + Q.n + 3 * wt / 4;
          len = (lane < 16 ? kAttnRowWords : 3 * kAttnRowWords / 4) * kRows;
          dst = lane < 16 ? stage + t * kAttnLowPitch : stage + kAttnCodesOffset + t * kAttnCodePitch;
        } else if (mode == 6 && lane < 16 && copies) {
          off = 1 + 2 * wt;
          len = 2 * kAttnRowWords * kRows;
          dst = stage + t * kAttnRawPitch;
        } else if (kTop16 && mode == 5 && copies) {  // body rows, nibble rows
          off = lane < 16 ? 5 + wt : 5 + Q.n + wt / 2;
          len = (lane < 16 ? kAttnRowWords : kAttnRowWords / 2) * kRows;
          dst = lane < 16 ? stage + t * kAttnLowPitch : stage + kAttnCodesOffset + t * kAttnNibblePitch;
        }
        const RowCopy c = plan_row_copy(Q.stream, Q.stream_bytes, off, len);
        const uint32_t total = warp_sum(c.bulk);
        if (lane == 0 && total > 0) mbar_expect_tx(&R.full[p.s], total);
        __syncwarp();
        issue_row_copy(c, dst, &R.full[p.s]);
        const uint32_t pad = c.pad;
        const uint32_t pad_y = __shfl_sync(kFull, pad, 16);
        if (lane == 0) {
          d.item = item;
          d.block = blk;
          d.plane = plane;
          d.mode = mode;
          d.pad_x = pad;
          d.pad_y = (mode == 3 || mode == 5) ? pad_y : 0u;
          const uint32_t first = blk * kAttnBlockTokens;
          d.valid = Q.ctx > first ? min(Q.ctx - first, static_cast<uint32_t>(kAttnBlockTokens)) : 0u;
        }
        if (mode != 5) reinterpret_cast<uint16_t*>(d.pal)[lane] = static_cast<uint16_t>(pal);
        __syncwarp();  // the lanes' palette, escape and edge-byte stores precede lane 0's release
        if (lane == 0) mbar_arrive(&R.full[p.s]);
        p.next();
      }
    }
    return;
  }

  if (kTop16 && warp == kAttnConsumerWarps + 1) {
    // ------------------------------------------------------- escape warp
    // For each stage of a top16 item: the block plane's escapes from the
    // stream's sorted entries, written into the stage's tail while the
    // producer stages the next copies.  It takes the stages in the
    // producer's order, waits for their release like the producer, and is
    // the second arrival on every stage's full barrier.
    AttnPos p;
    for (uint32_t item = i_begin; item < i_end; ++item) {
      const AttnItem& I = b.item[item];
      const AttnReq& Q = b.req[I.req];
      uint32_t mode = __ldg(Q.stream);
      const uint64_t cap = (Q.n + 199) / 200;
      if (mode != 5 || Q.tables == nullptr || 5 + Q.n + (Q.n + 1) / 2 + 5 * cap > Q.stream_bytes) mode = 0;
      // the entries (sorted by position) and a cursor at the first entry
      // of the item's first K block
      const uint8_t* entries = Q.stream + 5 + Q.n + (Q.n + 1) / 2;
      uint32_t esc_total = 0, cursor = 0;
      uint32_t books = 0;  // lanes 0-15: the K plane's book
      if (mode == 5) {
        esc_total = static_cast<uint32_t>(min(static_cast<uint64_t>(load_u32le(Q.stream + 1)), cap));
        cursor = entries_lower_bound(entries, esc_total, static_cast<uint64_t>(I.block0) * kAttnBlockWords);
        books = __ldg(Q.tables + 512 + (lane & 15));
      }
      for (uint32_t k = 0; k < 2 * I.blocks; ++k) {
        const uint32_t blk = I.block0 + (k >> 1), plane = k & 1;
        producer_acquire(R, p, nullptr);
        uint8_t* stage = ring + p.s * kAttnStageBytes;
        if (mode == 5 && plane == 0) {
          // K plane: the K warps decode an escaped word from its book
          // exponent like any other word; the difference between its true
          // and its book value times q, summed per token and q head, is
          // their correction of S^T.  Chunks of 32 entries from the cursor,
          // each lane one entry, summed over runs of equal (token, kv head)
          // (the entries are sorted by position).
          const uint64_t w_start = static_cast<uint64_t>(blk) * kAttnBlockWords;
          const uint32_t first = cursor;
          float4* zero = reinterpret_cast<float4*>(stage + kAttnEscCorr);
#pragma unroll
          for (int z = 0; z < static_cast<int>(kAttnCorrBytes / 16 / 32); ++z)
            zero[lane + 32 * z] = make_float4(0.f, 0.f, 0.f, 0.f);
          __syncwarp();
          float* cs = reinterpret_cast<float*>(stage + kAttnEscCorr);
          const uint32_t group = b.group;
          uint32_t count = 0;
          for (;;) {
            const uint32_t i = first + count + lane;
            uint64_t at = ~0ull;
            uint32_t ex = 0;
            if (i < esc_total) {
              at = entry_pos(entries, i) - w_start;
              ex = __ldg(entries + 5ull * i + 4);
            }
            const bool in = i < esc_total && at < kAttnBlockWords;
            const uint32_t bal = __ballot_sync(kFull, in);
            if ((bal & (bal + 1)) != 0 && lane == 0) raise_error(nullptr);  // entries out of order
            uint32_t body = 0, nib = 0;
            if (in) {
              const uint64_t w = w_start + at;
              body = __ldg(Q.stream + 5 + w);
              nib = (static_cast<uint32_t>(__ldg(Q.stream + 5 + Q.n + (w >> 1))) >> (4 * static_cast<uint32_t>(w & 1))) & 15u;
            }
            const uint32_t bexp = __shfl_sync(kFull, books, nib) & 0xFFu;
            const float delta = in ? top16_value(body, ex) - top16_value(body, bexp) : 0.f;
            const uint32_t key = in ? static_cast<uint32_t>(at >> 7) : 0xFFFFFFFFu;  // token * 8 + kv head
            const uint32_t hk = key & 7u, t = (key >> 3) & 15u, dl = static_cast<uint32_t>(at) & 127u;
            // the scan steps that stay inside the lane's run, and the run's last lane
            uint32_t same = 0;
#pragma unroll
            for (int s = 0; s < 5; ++s) {
              const uint32_t k2 = __shfl_up_sync(kFull, key, 1u << s);
              if (lane >= (1u << s) && k2 == key) same |= 1u << s;
            }
            const uint32_t knext = __shfl_down_sync(kFull, key, 1);
            const bool last = in && (lane == 31 || knext != key);
            const uint16_t* qrow = Q.q + static_cast<uint64_t>(hk) * group * kAttnHeadDim + dl;
            float qv[kAttnMaxGroup];
#pragma unroll
            for (int q = 0; q < kAttnMaxGroup; ++q)
              qv[q] = in && q < static_cast<int>(group)
                          ? __uint_as_float(static_cast<uint32_t>(__ldg(qrow + q * kAttnHeadDim)) << 16)
                          : 0.f;
#pragma unroll
            for (int q = 0; q < kAttnMaxGroup; ++q) {
              if (q >= static_cast<int>(group)) break;
              float v = delta * qv[q];
#pragma unroll
              for (int s = 0; s < 5; ++s) {
                const float u = __shfl_up_sync(kFull, v, 1u << s);
                if ((same >> s) & 1u) v += u;
              }
              if (last) cs[corr_index(t, hk, q)] += v;
            }
            __syncwarp();  // a run that continues in the next chunk adds to this chunk's sum
            count += __popc(bal);
            if (bal != kFull) break;
          }
          cursor = first + count;
        }  // V stages: their escapes are added to the items' partials by AttnEscapeKernel
        __syncwarp();  // the lanes' stores of the stage's share precede lane 0's arrival
        if (lane == 0) mbar_arrive(&R.full[p.s]);
        p.next();
      }
    }
    return;
  }

  const uint32_t gid = lane >> 2;  // MMA group
  const uint32_t tig = lane & 3;   // thread in group
  const uint32_t head = warp & (kAttnKvHeads - 1);
  const uint32_t group = b.group;
  AttnHandoff& H = hand[head];
  const uint8_t* pairs = reinterpret_cast<const uint8_t*>(pair);
  int pair_req = -1;

  if (warp < kAttnKvHeads) {
    // ------------------------------------------------------------ K warps
    // S^T = K Q^T over the K plane blocks (even ring positions).  The k
    // index of the MMAs runs over the head's dims in a lane-friendly order:
    // k slots 2 tig + {0, 1} of step kk are dims 32 tig + 4 kk + {0, 1}, k
    // slots 2 tig + 8 + {0, 1} are dims 32 tig + 4 kk + {2, 3}, in both K
    // and Q, so each lane decodes 32 consecutive dims of tokens gid, gid + 8.
    uint32_t fills = 0;  // S^T fragments handed over
    AttnPos p;
    for (uint32_t item = i_begin; item < i_end; ++item) {
      const AttnItem& I = b.item[item];
      const int req = static_cast<int>(I.req);
      if (req != pair_req) {
        // the request's pair table: every consumer warp is past the previous
        // item.  fixed6: from the palette of the item's first stage; top16:
        // per plane, the book exponents of a code byte's two words at their
        // places in a word pair (bits 7 and 23), 256 entries a plane
        attn_consumer_sync();
        consumer_wait(R, p, nullptr);
        if (kTop16 && D[p.s].mode == 5) {
          const uint8_t* books = b.req[I.req].tables + 512;
          for (int i = tid; i < 512; i += kAttnKThreads) {
            const uint8_t* bk = books + 16 * (i >> 8);
            pair[i] = (static_cast<uint32_t>(__ldg(bk + (i & 15))) << 7) |
                      (static_cast<uint32_t>(__ldg(bk + ((i >> 4) & 15))) << 23);
          }
        } else {
          const uint8_t* pal = D[p.s].pal;
          for (int i = tid; i < 4096; i += kAttnKThreads) pair[i] = pair_entry(pal, i);
        }
        pair_req = req;
        attn_consumer_sync();
      }
      uint32_t qb[16];  // Q[q head gid][dims 32 tig + 2i, +1]
      {
        const uint32_t* qh = reinterpret_cast<const uint32_t*>(
            b.req[I.req].q + static_cast<uint64_t>(head * group + gid) * kAttnHeadDim + 32 * tig);
#pragma unroll
        for (int i = 0; i < 16; ++i) qb[i] = gid < group ? qh[i] : 0u;
      }
      for (uint32_t blk = 0; blk < I.blocks; ++blk, ++fills) {
        consumer_wait(R, p, nullptr);
        const AttnDesc& d = D[p.s];
        const uint8_t* stage = ring + p.s * kAttnStageBytes;
        float sc[4] = {0.f, 0.f, 0.f, 0.f}, sd[4] = {0.f, 0.f, 0.f, 0.f};  // even / odd steps
        const uint32_t dim = head * kAttnHeadDim + 32 * tig;
        if (d.mode == 3) {
          uint32_t L0[8], C0[6], L1[8], C1[6];
          fixed6_load<16>(d, stage, gid, dim, L0, C0);
          fixed6_load<16>(d, stage, gid + 8, dim, L1, C1);
#pragma unroll
          for (int kk = 0; kk < 8; ++kk)
            mma_bf16((kk & 1) ? sd : sc, fixed6_word_pair<16>(pairs, L0, C0, 2 * kk),
                     fixed6_word_pair<16>(pairs, L1, C1, 2 * kk), fixed6_word_pair<16>(pairs, L0, C0, 2 * kk + 1),
                     fixed6_word_pair<16>(pairs, L1, C1, 2 * kk + 1), qb[2 * kk], qb[2 * kk + 1]);
        } else if (d.mode == 6) {
#pragma unroll
          for (int kk = 0; kk < 8; ++kk)
            mma_bf16((kk & 1) ? sd : sc, raw_word_pair(d, stage, gid, dim, 2 * kk),
                     raw_word_pair(d, stage, gid + 8, dim, 2 * kk), raw_word_pair(d, stage, gid, dim, 2 * kk + 1),
                     raw_word_pair(d, stage, gid + 8, dim, 2 * kk + 1), qb[2 * kk], qb[2 * kk + 1]);
        } else if (kTop16 && d.mode == 5) {
          const uint32_t* t16 = pair;  // the K plane's code-byte table
          uint32_t B0[8], N0[4], B1[8], N1[4];
          top16_load<16>(d, stage, gid, dim, B0, N0);
          top16_load<16>(d, stage, gid + 8, dim, B1, N1);
#pragma unroll
          for (int kk = 0; kk < 8; ++kk) {
            const uint32_t n0 = N0[kk >> 1] >> (16 * (kk & 1)), n1 = N1[kk >> 1] >> (16 * (kk & 1));
            const uint32_t a0 = top16_pair_t(B0[kk], t16[n0 & 0xFFu], false);
            const uint32_t a2 = top16_pair_t(B0[kk], t16[(n0 >> 8) & 0xFFu], true);
            const uint32_t a1 = top16_pair_t(B1[kk], t16[n1 & 0xFFu], false);
            const uint32_t a3 = top16_pair_t(B1[kk], t16[(n1 >> 8) & 0xFFu], true);
            mma_bf16((kk & 1) ? sd : sc, a0, a1, a2, a3, qb[2 * kk], qb[2 * kk + 1]);
          }
          // the escapes' share, from the escape warp: (gid, 2 tig .. +1) and (gid + 8, ..)
          const float* cs = reinterpret_cast<const float*>(stage + kAttnEscCorr);
          const float2 e0 = *reinterpret_cast<const float2*>(cs + corr_index(gid, head, 2 * tig));
          const float2 e1 = *reinterpret_cast<const float2*>(cs + corr_index(gid + 8, head, 2 * tig));
          sc[0] += e0.x;
          sc[1] += e0.y;
          sc[2] += e1.x;
          sc[3] += e1.y;
        }  // else: a stream this kernel does not read (the producer raised an error): S^T = 0
        const uint32_t valid = d.valid;
        consumer_release(R, p);
        p.next();
        p.next();
        // hand S^T to the V warp of the head
        const uint32_t slot = fills & 1, use = fills >> 1;
        if (use > 0) wait_stage(&H.empty[slot], (use - 1) & 1, nullptr);
        scores[head][slot][lane] = make_float4(sc[0] + sd[0], sc[1] + sd[1], sc[2] + sd[2], sc[3] + sd[3]);
        if (lane == 0) H.valid[slot] = valid;
        __syncwarp();
        if (lane == 0) mbar_arrive(&H.full[slot]);
      }
    }
    return;
  }

  // -------------------------------------------------------------- V warps
  // Softmax of S^T and O^T += V^T P^T over the V plane blocks (odd ring
  // positions).  The M index of the MMAs runs over the head's dims in a
  // lane-friendly order: rows gid, gid + 8 of step m are dims 16 gid + 2m,
  // +1, so each lane decodes 16 consecutive dims of tokens 2 tig, 2 tig + 1,
  // 2 tig + 8, 2 tig + 9 and the k pairs of the A fragments come from
  // byte permutes of two tokens' word pairs.
  uint32_t uses = 0;  // S^T fragments taken
  AttnPos p;
  p.next();
  for (uint32_t item = i_begin; item < i_end; ++item) {
    const AttnItem& I = b.item[item];
    const int req = static_cast<int>(I.req);
    if (req != pair_req) {  // the K warps rebuild the pair table in between
      attn_consumer_sync();
      pair_req = req;
      attn_consumer_sync();
    }
    float o[8][4];  // O^T: (dim 16 gid + 2m, head 2 tig), (.., 2 tig + 1), (dim + 1, 2 tig), (dim + 1, 2 tig + 1)
#pragma unroll
    for (int m = 0; m < 8; ++m) o[m][0] = o[m][1] = o[m][2] = o[m][3] = 0.f;
    float mx[2] = {-INFINITY, -INFINITY}, lsum[2] = {0.f, 0.f};
    for (uint32_t blk = 0; blk < I.blocks; ++blk, ++uses) {
      const uint32_t slot = uses & 1;
      wait_stage(&H.full[slot], (uses >> 1) & 1, nullptr);
      const float4 s4 = scores[head][slot][lane];
      const uint32_t valid = H.valid[slot];
      __syncwarp();
      if (lane == 0) mbar_arrive(&H.empty[slot]);
      // ---- online softmax per q head (column) over tokens gid, gid + 8 of all lanes with this tig
      float x[4];
      x[0] = gid < valid ? s4.x * b.scale_log2 : -INFINITY;
      x[1] = gid < valid ? s4.y * b.scale_log2 : -INFINITY;
      x[2] = gid + 8 < valid ? s4.z * b.scale_log2 : -INFINITY;
      x[3] = gid + 8 < valid ? s4.w * b.scale_log2 : -INFINITY;
      float pe[4], alpha[2];
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        float bm = fmaxf(x[e], x[2 + e]);
        bm = fmaxf(bm, __shfl_xor_sync(kFull, bm, 4));
        bm = fmaxf(bm, __shfl_xor_sync(kFull, bm, 8));
        bm = fmaxf(bm, __shfl_xor_sync(kFull, bm, 16));
        const float m_new = fmaxf(mx[e], bm);
        alpha[e] = exp2f(mx[e] - m_new);  // 0 on the first block (mx = -inf)
        pe[e] = exp2f(x[e] - m_new);
        pe[2 + e] = exp2f(x[2 + e] - m_new);
        float bs = pe[e] + pe[2 + e];
        bs += __shfl_xor_sync(kFull, bs, 4);
        bs += __shfl_xor_sync(kFull, bs, 8);
        bs += __shfl_xor_sync(kFull, bs, 16);
        lsum[e] = lsum[e] * alpha[e] + bs;
        mx[e] = m_new;
      }
      if (!__all_sync(kFull, alpha[0] == 1.f && alpha[1] == 1.f)) {  // a running max moved
#pragma unroll
        for (int m = 0; m < 8; ++m) {
          o[m][0] *= alpha[0];
          o[m][1] *= alpha[1];
          o[m][2] *= alpha[0];
          o[m][3] *= alpha[1];
        }
      }
      // P^T rows (tokens gid, gid+8) x head pairs -> B fragments of V^T P^T
      const uint32_t h0 = pack_bf16(pe[0], pe[1]), h1 = pack_bf16(pe[2], pe[3]);
      const uint32_t l0 = pack_bf16(pe[0] - __uint_as_float(h0 << 16), pe[1] - __uint_as_float(h0 & 0xFFFF0000u));
      const uint32_t l1 = pack_bf16(pe[2] - __uint_as_float(h1 << 16), pe[3] - __uint_as_float(h1 & 0xFFFF0000u));
      const uint32_t ph0 = movmatrix_trans(h0), ph1 = movmatrix_trans(h1);
      const uint32_t pl0 = movmatrix_trans(l0), pl1 = movmatrix_trans(l1);
      // ---- O^T += V^T P^T
      consumer_wait(R, p, nullptr);
      {
        const AttnDesc& d = D[p.s];
        const uint8_t* stage = ring + p.s * kAttnStageBytes;
        const uint32_t dim = head * kAttnHeadDim + 16 * gid;
        // tokens 2 tig, 2 tig + 1, 2 tig + 8, 2 tig + 9; words past the
        // context may hold anything (P is 0 there) and are read as 0
        const uint32_t t0 = 2 * tig, t2 = 2 * tig + 8;
        const bool k0 = t0 < valid, k1 = t0 + 1 < valid, k2 = t2 < valid, k3 = t2 + 1 < valid;
        auto mma_step = [&](int m, uint32_t v0, uint32_t v1, uint32_t v2, uint32_t v3) {
          v0 = k0 ? v0 : 0u;
          v1 = k1 ? v1 : 0u;
          v2 = k2 ? v2 : 0u;
          v3 = k3 ? v3 : 0u;
          const uint32_t a0 = __byte_perm(v0, v1, 0x5410), a1 = __byte_perm(v0, v1, 0x7632);
          const uint32_t a2 = __byte_perm(v2, v3, 0x5410), a3 = __byte_perm(v2, v3, 0x7632);
          mma_bf16(o[m], a0, a1, a2, a3, ph0, ph1);
          mma_bf16(o[m], a0, a1, a2, a3, pl0, pl1);
        };
        if (d.mode == 3) {
          uint32_t L0[4], C0[3], L1[4], C1[3], L2[4], C2[3], L3[4], C3[3];
          fixed6_load<8>(d, stage, t0, dim, L0, C0);
          fixed6_load<8>(d, stage, t0 + 1, dim, L1, C1);
          fixed6_load<8>(d, stage, t2, dim, L2, C2);
          fixed6_load<8>(d, stage, t2 + 1, dim, L3, C3);
#pragma unroll
          for (int m = 0; m < 8; ++m)
            mma_step(m, fixed6_word_pair<8>(pairs, L0, C0, m), fixed6_word_pair<8>(pairs, L1, C1, m),
                     fixed6_word_pair<8>(pairs, L2, C2, m), fixed6_word_pair<8>(pairs, L3, C3, m));
        } else if (d.mode == 6) {
#pragma unroll
          for (int m = 0; m < 8; ++m)
            mma_step(m, raw_word_pair(d, stage, t0, dim, m), raw_word_pair(d, stage, t0 + 1, dim, m),
                     raw_word_pair(d, stage, t2, dim, m), raw_word_pair(d, stage, t2 + 1, dim, m));
        } else if (kTop16 && d.mode == 5) {
          const uint32_t* t16 = pair + 256;  // the V plane's code-byte table
          const uint32_t tok[4] = {t0, t0 + 1, t2, t2 + 1};
          uint32_t B[4][4], N[4][2];
#pragma unroll
          for (int j = 0; j < 4; ++j) top16_load<8>(d, stage, tok[j], dim, B[j], N[j]);
#pragma unroll
          for (int m = 0; m < 8; ++m) {
            uint32_t v[4];
#pragma unroll
            for (int j = 0; j < 4; ++j)
              v[j] = top16_pair_t(B[j][m >> 1], t16[(N[j][m >> 2] >> (8 * (m & 3))) & 0xFFu], (m & 1) != 0);
            mma_step(m, v[0], v[1], v[2], v[3]);
          }
          // the block's scaled scores (masked past the context), for the
          // escapes' correction: [kv head][token][q head slot] of the block
          float* sx = b.scores + (static_cast<uint64_t>(I.gblock0 + blk) * kAttnKvHeads + head) *
                                     kAttnBlockTokens * group;
#pragma unroll
          for (int e = 0; e < 2; ++e) {
            const uint32_t col = 2 * tig + e;
            if (col < group) {
              sx[gid * group + col] = x[e];
              sx[(gid + 8) * group + col] = x[2 + e];
            }
          }
        }
      }
      consumer_release(R, p);
      p.next();
      p.next();
    }
    // partial of the item: O^T columns of the group's heads (dims 16 gid .. 16 gid + 15 per lane), m and l
    float* base = b.partials + static_cast<uint64_t>(item) * kAttnKvHeads * group * kAttnRecord;
#pragma unroll
    for (int e = 0; e < 2; ++e) {
      const uint32_t hcol = 2 * tig + e;
      if (hcol < group) {
        float* dst = base + static_cast<uint64_t>(head * group + hcol) * kAttnRecord;
        float4* row = reinterpret_cast<float4*>(dst + 16 * gid);
#pragma unroll
        for (int j = 0; j < 4; ++j)
          row[j] = make_float4(o[2 * j][e], o[2 * j][2 + e], o[2 * j + 1][e], o[2 * j + 1][2 + e]);
        if (gid == 0) {
          dst[kAttnHeadDim] = mx[e];
          dst[kAttnHeadDim + 1] = lsum[e];
        }
      }
    }
  }
}

// V-plane escapes of top16 streams.  The V warps decode an escaped V word
// from its book exponent, so each q head's partial O of the item lacks
// p * delta at the word's dim: delta = true - book value of the word, p =
// 2^(x - m) the weight of the word's token in the partial's scale (x the
// token's scaled score, saved by the V warps; m the partial's running max).
// One CTA per item, in batches of the item's V escapes:
//   - two warps find the item's V escapes by searches of the sorted entries;
//   - every thread computes the shares of a few escapes (four at a time, so
//     that their loads overlap) into shared memory;
//   - warp h adds those of kv head h to the item's sums in shared memory,
//     [q head][dim], 32 entries at a time: the lanes of entries with the
//     same dim take turns in lane order, so a sum takes its terms in entry
//     order;
//   - at the end warp h adds its head's sums to the partials.
// Every run adds the same terms in the same order (no atomics).
constexpr uint32_t kAttnEscSmem = 96 * 1024;        // dynamic shared bytes: sums, then a batch
constexpr int kAttnEscThreads = 64 * kAttnKvHeads;  // 16 warps; warps 0-7 also add the shares
static_assert(kAttnKvHeads * kAttnMaxGroup * kAttnHeadDim * 4 + 4096 * 6 <= kAttnEscSmem, "escape batch room");

template <int kMaxR, int kMaxI>
__global__ void __launch_bounds__(kAttnEscThreads, 2) AttnEscapeKernel(const __grid_constant__ AttnBatch<kMaxR, kMaxI> b) {
  extern __shared__ __align__(16) uint8_t esm[];
  __shared__ uint32_t range[2];
  __shared__ float mq[kAttnKvHeads * kAttnMaxGroup];  // the item's running max per q head
  const uint32_t item = blockIdx.x;
  if (item >= b.items) return;
  const AttnItem& I = b.item[item];
  const AttnReq& Q = b.req[I.req];
  if (Q.tables == nullptr) return;
  const uint64_t cap = (Q.n + 199) / 200;
  // a stream the attention kernel did not read as top16 (it raised the error)
  if (__ldg(Q.stream) != 5 || 5 + Q.n + (Q.n + 1) / 2 + 5 * cap > Q.stream_bytes) return;
  const uint8_t* entries = Q.stream + 5 + Q.n + (Q.n + 1) / 2;
  const uint32_t esc_total = static_cast<uint32_t>(min(static_cast<uint64_t>(load_u32le(Q.stream + 1)), cap));
  const uint64_t half = Q.n / 2;  // the V plane's first word
  const uint64_t v0 = half + static_cast<uint64_t>(I.block0) * kAttnBlockWords;
  const uint64_t v1 = v0 + static_cast<uint64_t>(I.blocks) * kAttnBlockWords;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  constexpr uint32_t T = kAttnEscThreads;
  const uint32_t group = b.group, heads = kAttnKvHeads * group;
  float* partial = b.partials + static_cast<uint64_t>(item) * heads * kAttnRecord;
  if (warp < 2) {
    const uint32_t r = entries_lower_bound(entries, esc_total, warp == 0 ? v0 : v1);
    if (lane == 0) range[warp] = r;
  }
  float* sums = reinterpret_cast<float*>(esm);  // [q head][dim]
  for (uint32_t i = tid; i < heads * kAttnHeadDim; i += T) sums[i] = 0.f;
  if (static_cast<uint32_t>(tid) < heads) mq[tid] = partial[tid * kAttnRecord + kAttnHeadDim];
  __syncthreads();
  const uint32_t lo = range[0], hi = range[1];
  if (lo >= hi) return;
  // the batch: entries that fit the rest as a u16 key and `group` shares each
  const uint32_t room = kAttnEscSmem - heads * kAttnHeadDim * 4;
  const uint32_t batch = min(4096u, (room - 16) / (2 + 4 * group) / 256 * 256);
  uint16_t* skey = reinterpret_cast<uint16_t*>(esm + heads * kAttnHeadDim * 4);  // kv head << 7 | dim, or 0xFFFF
  float* sval = reinterpret_cast<float*>(esm + heads * kAttnHeadDim * 4 + ((2 * batch + 15) & ~15u));
  const uint8_t* vbook = Q.tables + 528;
  for (uint32_t e0 = lo; e0 < hi; e0 += batch) {
    const uint32_t cnt = min(hi - e0, batch);
    for (uint32_t k0 = 0; k0 < cnt; k0 += 4 * T) {
      uint32_t kk[4], key[4], ex[4], body[4], nb[4];
      uint64_t pos[4];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        kk[j] = k0 + T * j + tid;
        pos[j] = kk[j] < cnt ? entry_pos(entries, e0 + kk[j]) : v1;
      }
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        key[j] = 0xFFFFu;
        if (kk[j] < cnt && (pos[j] < v0 || pos[j] >= v1)) raise_error(nullptr);  // entries out of order
        if (pos[j] >= v0 && pos[j] < v1) {
          const uint32_t wv = static_cast<uint32_t>(pos[j] - v0);  // word of the item's V blocks
          if (I.block0 * kAttnBlockTokens + wv / kAttnRowWords < Q.ctx) {  // words past the context are read as 0
            key[j] = wv % kAttnRowWords;  // kv head << 7 | dim
            ex[j] = __ldg(entries + 5ull * (e0 + kk[j]) + 4);
            body[j] = __ldg(Q.stream + 5 + pos[j]);
            nb[j] = __ldg(Q.stream + 5 + Q.n + (pos[j] >> 1));
          }
        }
      }
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        if (key[j] != 0xFFFFu) {
          const uint32_t wv = static_cast<uint32_t>(pos[j] - v0);
          const uint32_t hk = key[j] >> 7;
          const uint32_t nib = (nb[j] >> (4 * static_cast<uint32_t>(pos[j] & 1))) & 15u;
          const float delta = top16_value(body[j], ex[j]) - top16_value(body[j], __ldg(vbook + nib));
          // scores of the token: [batch block][kv head][token][q head slot]
          const float* xs = b.scores + ((static_cast<uint64_t>(I.gblock0 + wv / kAttnBlockWords) * kAttnKvHeads + hk) *
                                            kAttnBlockTokens + (wv / kAttnRowWords) % kAttnBlockTokens) * group;
          float xv[kAttnMaxGroup];
#pragma unroll
          for (int q = 0; q < kAttnMaxGroup; ++q) xv[q] = q < static_cast<int>(group) ? xs[q] : 0.f;
#pragma unroll
          for (int q = 0; q < kAttnMaxGroup; ++q)
            if (q < static_cast<int>(group)) sval[kk[j] * group + q] = exp2f(xv[q] - mq[hk * group + q]) * delta;
        }
        if (kk[j] < cnt) skey[kk[j]] = static_cast<uint16_t>(key[j]);
      }
    }
    __syncthreads();
    if (warp < kAttnKvHeads) {
      // kv head `warp`: 32 entries at a time, the lanes of one dim in turn
      for (uint32_t c = 0; c < cnt; c += 32) {
        const uint32_t key = c + lane < cnt ? skey[c + lane] : 0xFFFFu;
        const bool mine = (key >> 7) == static_cast<uint32_t>(warp);
        if (__ballot_sync(kFull, mine) == 0) continue;
        const uint32_t dl = key & 127u;
        const uint32_t peers = __match_any_sync(kFull, mine ? dl : 128u + lane);
        const uint32_t rank = __popc(peers & ((1u << lane) - 1u));
        const uint32_t turns = __reduce_max_sync(kFull, mine ? rank : 0u);
        for (uint32_t t = 0; t <= turns; ++t) {
          if (mine && rank == t) {
            const float* v = sval + (c + lane) * group;
            float* dst = sums + warp * group * kAttnHeadDim + dl;
            for (uint32_t q = 0; q < group; ++q) dst[q * kAttnHeadDim] += v[q];
          }
          __syncwarp();
        }
      }
    }
    __syncthreads();  // the batch is read before the next one is written
  }
  if (warp < kAttnKvHeads) {
    float* o = partial + static_cast<uint64_t>(warp) * group * kAttnRecord + 4 * lane;
    const float* sm = sums + warp * group * kAttnHeadDim + 4 * lane;
    for (uint32_t q = 0; q < group; ++q) {
      const float4 a = *reinterpret_cast<const float4*>(sm + q * kAttnHeadDim);
      float4 r = *reinterpret_cast<float4*>(o + q * kAttnRecord);
      r.x += a.x;
      r.y += a.y;
      r.z += a.z;
      r.w += a.w;
      *reinterpret_cast<float4*>(o + q * kAttnRecord) = r;
    }
  }
}

// Merge the items of every request: out = sum_i 2^(m_i - M) o_i / sum_i 2^(m_i - M) l_i.
// One warp per (request, q head): the items' (m, l) are read across lanes,
// then each lane accumulates 4 dims over the items.
template <int kMaxR, int kMaxI>
__global__ void __launch_bounds__(256) AttnCombineKernel(const __grid_constant__ AttnBatch<kMaxR, kMaxI> b) {
  const uint32_t heads = kAttnKvHeads * b.group;
  const uint32_t wid = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (wid >= b.reqs * heads) return;
  const AttnReq& Q = b.req[wid / heads];
  const uint32_t hq = wid % heads;
  // records of the request: one per item
  auto rec = [&](uint32_t i) {
    return b.partials + (static_cast<uint64_t>(Q.first_item + i) * heads + hq) * kAttnRecord;
  };
  const uint32_t records = Q.items;
  float M = -INFINITY;
  for (uint32_t i = lane; i < records; i += 32) M = fmaxf(M, rec(i)[kAttnHeadDim]);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) M = fmaxf(M, __shfl_xor_sync(kFull, M, o));
  float L = 0.f;
  float acc[4] = {0.f, 0.f, 0.f, 0.f};
  for (uint32_t i0 = 0; i0 < records; i0 += 32) {
    // weights of 32 records across the lanes, then their O rows accumulated
    const uint32_t mine = i0 + lane;
    const float w_l = mine < records ? exp2f(rec(mine)[kAttnHeadDim] - M) : 0.f;
    L += mine < records ? w_l * rec(mine)[kAttnHeadDim + 1] : 0.f;
    const uint32_t n = min(32u, records - i0);
#pragma unroll 4
    for (uint32_t j = 0; j < n; ++j) {
      const float w = __shfl_sync(kFull, w_l, j);
      const float4 v = *reinterpret_cast<const float4*>(rec(i0 + j) + 4 * lane);
      acc[0] += w * v.x;
      acc[1] += w * v.y;
      acc[2] += w * v.z;
      acc[3] += w * v.w;
    }
  }
  L = warp_sum(L);
  const float inv = 1.f / L;
  uint16_t* dst = Q.out + static_cast<uint64_t>(hq) * kAttnHeadDim + 4 * lane;
  *reinterpret_cast<uint2*>(dst) =
      make_uint2(pack_bf16(acc[0] * inv, acc[1] * inv), pack_bf16(acc[2] * inv, acc[3] * inv));
}

}  // namespace ukv
