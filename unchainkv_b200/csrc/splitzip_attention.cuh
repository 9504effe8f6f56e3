// Codec-aware GQA decode attention over splitzip streams (sm_100a).
//
// One decode query per request attends over that request's K/V of one layer,
// read straight from the request's transfer stream (the codec's output for
// the request's paged blocks, K plane then V plane) without decoding it into
// a paged cache first.  The reference receiver instead decodes the stream
// into its cache and runs attention on the bf16 copy.
//
// Shape (the Llama-3-8B decode of the benchmark configuration): 8 kv heads x
// 128 dims, 16-token blocks, GQA group g <= 16 q heads per kv head.
//
// Work: the blocks of all requests, in order, are split evenly over the
// persistent CTAs; an item is one CTA's run of blocks of one request (a CTA
// holds one or a few items).  Per item:
//   - producer warp: for each block, stages the K plane block (16 tokens x
//     8 heads x 128 dims), then the V plane block, into a ring of shared
//     memory stages by TMA (the stream regions of that block's words: the
//     low-byte plane and 6-bit codes for fixed6, the words for raw);
//   - decoder warp h (kv head h): decodes its head's 16 x 128 slice of every
//     staged plane block into a swizzled bf16 tile in shared memory (a K
//     slot and a V slot per head) and releases the stage;
//   - MMA warp h: computes S^T = K Q^T (16 tokens x g q heads) on one
//     m16n8k16 bf16 MMA per 16 dims with K fragments from ldmatrix, keeps an
//     online softmax per q head in fp32 (base 2), turns P^T into the PV
//     operand in registers (movmatrix), and accumulates O^T += V^T P^T
//     (128 dims x g) with V^T fragments from ldmatrix.trans; P is split into
//     two bf16 parts (hi + lo) so that large V values do not amplify its
//     rounding.  Decoder and MMA warp of a head hand the slots over with
//     full/empty mbarriers, so decoding and MMAs overlap;
//   - every item writes a partial (m, l, O) per q head to a workspace and
//     AttnCombineKernel merges them per request.
// The tiles have g useful columns of 8 (g = 4 for the benchmark), so they
// run on warp-level MMAs; the kernel is bound by the HBM read of the
// compressed K/V.
#pragma once

#include "splitzip_kernels.cuh"

namespace ukv {

constexpr int kAttnHeadDim = 128;
constexpr int kAttnBlockTokens = 16;
constexpr int kAttnKvHeads = kWarps;  // consumer warps of one block parity
constexpr int kAttnConsumerWarps = 2 * kAttnKvHeads;  // a decoder and an MMA warp per kv head
constexpr int kAttnConsumers = 32 * kAttnConsumerWarps;
constexpr int kAttnThreads = kAttnConsumers + 32;     // + the producer warp
constexpr int kAttnDecoders = 32 * kAttnKvHeads;      // threads of the decoder warps
constexpr uint32_t kAttnBlockWords = kAttnBlockTokens * kAttnKvHeads * kAttnHeadDim;  // per plane
constexpr int kAttnStages = 4;
constexpr uint32_t kAttnStageBytes = 2 * kAttnBlockWords + 64;  // raw words of one plane block + pads
constexpr uint32_t kAttnCodesOffset = kAttnBlockWords + 32;     // fixed6 codes inside a stage
constexpr uint32_t kAttnTileBytes = kAttnBlockTokens * kAttnHeadDim * 2;  // one warp's bf16 tile
// dynamic shared memory: the ring stages, then one tile per consumer warp
constexpr uint32_t kAttnSmemBytes = kAttnStages * kAttnStageBytes + kAttnConsumerWarps * kAttnTileBytes;
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
  uint32_t ctx;           // valid tokens (the last block may be partial)
  uint32_t first_item;
  uint32_t items;
  uint32_t pad;
};

struct AttnItem {
  uint32_t req;
  uint32_t block0;
  uint32_t blocks;
  uint32_t pad;
};

template <int kMaxR, int kMaxI>
struct AttnBatch {
  uint32_t reqs;
  uint32_t items;
  uint32_t group;      // q heads per kv head
  float scale_log2;    // softmax scale * log2(e)
  float* partials;     // [items][kv_heads * group][kAttnRecord] (o, then m, l)
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

__device__ __forceinline__ void ldmatrix_x4(uint32_t (&r)[4], const void* p) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(smem_addr(p)));
}

__device__ __forceinline__ void ldmatrix_x4_trans(uint32_t (&r)[4], const void* p) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(smem_addr(p)));
}

// Transpose an 8x8 bf16 matrix held in MMA fragment layout across the warp.
__device__ __forceinline__ uint32_t movmatrix_trans(uint32_t x) {
  uint32_t r;
  asm volatile("movmatrix.sync.aligned.m8n8.trans.b16 %0, %1;" : "=r"(r) : "r"(x));
  return r;
}

// Barrier of the attention kernel's decoder warps (named barrier 1).
__device__ __forceinline__ void attn_decoder_sync() {
  asm volatile("bar.sync 1, %0;" ::"n"(kAttnDecoders) : "memory");
}

// Tile hand-over between the decoder and the MMA warp of a head: slot 0
// holds K tiles, slot 1 V tiles; full[slot] when decoded, empty[slot] when
// the MMA warp is done with it.  `valid` carries the block's valid tokens.
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

// A warp's 16-token x 128-dim bf16 tile: rows of 16 chunks of 16 bytes, chunk
// c of row t stored at chunk c ^ (t & 7) ^ (c / 8).  ldmatrix reads 8 rows of
// one logical chunk without bank conflicts, and so does the decode's store of
// chunks 2g (g = 0..7) of one row: the c / 8 term moves the upper 4 onto the
// odd bank groups.
__device__ __forceinline__ uint8_t* tile_chunk(uint8_t* tile, uint32_t t, uint32_t c) {
  return tile + t * 256 + ((c ^ (t & 7) ^ (c >> 3)) << 4);
}

// Decode this warp's head slice of a staged plane block into its tile: 128
// units of 16 words (token t = u / 8, dims 16 * (u % 8)), 4 per lane.
__device__ __forceinline__ void attn_decode_tile(const AttnDesc& d, const uint8_t* stage, const uint8_t* pair,
                                                 uint8_t* tile, int head, int lane) {
  const bool aligned = (d.pad_x | d.pad_y) == 0;
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    const uint32_t u = lane + 32 * k;
    const uint32_t t = u >> 3, g = u & 7;
    const uint32_t w0 = t * (kAttnKvHeads * kAttnHeadDim) + head * kAttnHeadDim + 16 * g;  // word in the block
    uint32_t o[8];
    if (d.mode == 3) {
      uint32_t Lw[4];
      uint32_t Q[4];  // 12 code bytes
      if (aligned) {  // uniform: the stream regions start on 16-byte boundaries
        const uint4 l4 = *reinterpret_cast<const uint4*>(stage + w0);
        Lw[0] = l4.x; Lw[1] = l4.y; Lw[2] = l4.z; Lw[3] = l4.w;
        const uint32_t* c = reinterpret_cast<const uint32_t*>(stage + kAttnCodesOffset + 3 * w0 / 4);
        Q[0] = c[0]; Q[1] = c[1]; Q[2] = c[2]; Q[3] = 0;
      } else {
        smem_read16_window(stage, d.pad_x + w0, Lw);
        // 16-byte window reads keep each quarter warp on one row's banks
        smem_read16_window(stage + kAttnCodesOffset, d.pad_y + 3 * w0 / 4, Q);
      }
      uint32_t f[8];
      f[0] = pair_slot((Q[0] << 2) & 0x3FFCu);
      f[1] = pair_slot((Q[0] >> 10) & 0x3FFCu);
      f[2] = pair_slot(__funnelshift_r(Q[0], Q[1], 22) & 0x3FFCu);
      f[3] = pair_slot((Q[1] >> 2) & 0x3FFCu);
      f[4] = pair_slot((Q[1] >> 14) & 0x3FFCu);
      f[5] = pair_slot(__funnelshift_r(Q[1], Q[2], 26) & 0x3FFCu);
      f[6] = pair_slot((Q[2] >> 6) & 0x3FFCu);
      f[7] = pair_slot((Q[2] >> 18) & 0x3FFCu);
#pragma unroll
      for (int i = 0; i < 8; ++i)
        o[i] = __byte_perm(Lw[i >> 1], 0, (i & 1) ? 0x4342 : 0x4140) |
               *reinterpret_cast<const uint32_t*>(pair + f[i]);
    } else if (d.mode == 6) {  // raw
      if (aligned) {
        const uint4* r = reinterpret_cast<const uint4*>(stage + 2 * w0);
        const uint4 a = r[0], b2 = r[1];
        o[0] = a.x; o[1] = a.y; o[2] = a.z; o[3] = a.w;
        o[4] = b2.x; o[5] = b2.y; o[6] = b2.z; o[7] = b2.w;
      } else {
        smem_read_words<8>(stage, d.pad_x + 2 * w0, o);
      }
    } else {  // a stream this kernel does not read: zeros (the producer raised an error)
#pragma unroll
      for (int i = 0; i < 8; ++i) o[i] = 0u;
    }
    *reinterpret_cast<uint4*>(tile_chunk(tile, t, 2 * g)) = make_uint4(o[0], o[1], o[2], o[3]);
    *reinterpret_cast<uint4*>(tile_chunk(tile, t, 2 * g + 1)) = make_uint4(o[4], o[5], o[6], o[7]);
  }
}

template <int kMaxR, int kMaxI>
__global__ void __launch_bounds__(kAttnThreads, 1) AttnKernel(const __grid_constant__ AttnBatch<kMaxR, kMaxI> b) {
  extern __shared__ __align__(128) uint8_t ring[];
  __shared__ __align__(16) uint32_t pair[4096];
  __shared__ __align__(16) AttnDesc D[kAttnStages];
  __shared__ AttnRing R;  // empty barriers count the kWarps == kAttnKvHeads decoder warps
  __shared__ __align__(8) AttnHandoff hand[kAttnKvHeads];
  const int tid = threadIdx.x;
  const int lane = tid & 31;
  const int warp = tid >> 5;
  ring_init(R);
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
    // K then V of each block of each item of this CTA; the mode byte and the
    // palette of the item's stream are read once per item
    AttnPos p;
    for (uint32_t item = i_begin; item < i_end; ++item) {
      const AttnItem& I = b.item[item];
      const AttnReq& Q = b.req[I.req];
      uint32_t mode = __ldg(Q.stream);
      const uint64_t need = mode == 3 ? 65 + Q.n + 3 * ((Q.n + 3) / 4) : mode == 6 ? 1 + 2 * Q.n : 0;
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
        const uint64_t w0 = plane * (Q.n / 2) + static_cast<uint64_t>(blk) * kAttnBlockWords;
        uint8_t* stage = ring + p.s * kAttnStageBytes;
        if (lane == 0) {
          uint2 pad{0, 0};
          if (mode == 3) {
            pad.x = stage_bytes_one(Q.stream, Q.stream_bytes, 65 + w0, kAttnBlockWords, stage, &R.full[p.s]);
            pad.y = stage_bytes_one(Q.stream, Q.stream_bytes, 65 + Q.n + 3 * w0 / 4, 3 * kAttnBlockWords / 4,
                                    stage + kAttnCodesOffset, &R.full[p.s]);
          } else if (mode == 6) {
            pad.x = stage_bytes_one(Q.stream, Q.stream_bytes, 1 + 2 * w0, 2 * kAttnBlockWords, stage, &R.full[p.s]);
          }
          d.item = item;
          d.block = blk;
          d.plane = plane;
          d.mode = mode;
          d.pad_x = pad.x;
          d.pad_y = pad.y;
          const uint32_t first = blk * kAttnBlockTokens;
          d.valid = Q.ctx > first ? min(Q.ctx - first, static_cast<uint32_t>(kAttnBlockTokens)) : 0u;
        }
        reinterpret_cast<uint16_t*>(d.pal)[lane] = static_cast<uint16_t>(pal);
        producer_commit(R, p);
        p.next();
      }
    }
    return;
  }

  // ---------------------------------------------------------- decoder warps
  const int head = warp & (kAttnKvHeads - 1);
  uint8_t* tiles = ring + kAttnStages * kAttnStageBytes + head * 2 * kAttnTileBytes;  // K slot, V slot
  AttnHandoff& H = hand[head];
  if (warp < kAttnKvHeads) {
    int pair_req = -1;
    uint32_t fills = 0;  // tiles decoded into each slot so far (same for both)
    AttnPos p;
    for (uint32_t item = i_begin; item < i_end; ++item) {
      const AttnItem& I = b.item[item];
      const int req = static_cast<int>(I.req);
      if (req != pair_req) {
        // the request's fixed6 pair table, built by the decoder warps: all
        // are past their stages of the previous item; the palette comes from
        // the item's first stage
        attn_decoder_sync();
        consumer_wait(R, p, nullptr);
        const uint8_t* pal = D[p.s].pal;
        for (int i = tid; i < 4096; i += kAttnDecoders)
          pair[i] = pair_entry(pal, i);
        pair_req = req;
        attn_decoder_sync();
      }
      for (uint32_t k = 0; k < 2 * I.blocks; ++k) {
        const uint32_t slot = k & 1;
        consumer_wait(R, p, nullptr);
        const AttnDesc& d = D[p.s];
        if (fills > 0) wait_stage(&H.empty[slot], (fills - 1) & 1, nullptr);  // the MMA warp is done with it
        attn_decode_tile(d, ring + p.s * kAttnStageBytes, reinterpret_cast<const uint8_t*>(pair),
                         tiles + slot * kAttnTileBytes, head, lane);
        if (lane == 0) H.valid[slot] = d.valid;
        __syncwarp();
        if (lane == 0) mbar_arrive(&H.full[slot]);
        consumer_release(R, p);
        p.next();
        if (slot == 1) ++fills;
      }
    }
    return;
  }

  // -------------------------------------------------------------- MMA warps
  const uint32_t group = b.group;
  const uint32_t gid = lane >> 2;  // MMA group: token gid (+8) of S^T, dim 16m + gid (+8) of O^T
  const uint32_t tig = lane & 3;   // q heads 2*tig, 2*tig + 1 of the group (valid below `group`)
  const uint8_t* tileK = tiles;
  const uint8_t* tileV = tiles + kAttnTileBytes;
  uint32_t uses = 0;  // tiles consumed from each slot so far
  for (uint32_t item = i_begin; item < i_end; ++item) {
    const AttnItem& I = b.item[item];
    // Q^T fragments (B operand of S^T = K Q^T): Q[q head gid][dims 16k + 2*tig (+8)]
    uint32_t qb[8][2];
    {
      const uint16_t* qh = b.req[I.req].q + static_cast<uint64_t>(head * group + gid) * kAttnHeadDim;
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        qb[k][0] = gid < group ? *reinterpret_cast<const uint32_t*>(qh + 16 * k + 2 * tig) : 0u;
        qb[k][1] = gid < group ? *reinterpret_cast<const uint32_t*>(qh + 16 * k + 8 + 2 * tig) : 0u;
      }
    }
    float o[8][4];  // O^T per 16 dims: (dim 16m+gid, head 2tig), (.., 2tig+1), (dim +8, 2tig), (dim +8, 2tig+1)
#pragma unroll
    for (int m = 0; m < 8; ++m) o[m][0] = o[m][1] = o[m][2] = o[m][3] = 0.f;
    float mx[2] = {-INFINITY, -INFINITY}, lsum[2] = {0.f, 0.f};
    for (uint32_t blk = 0; blk < I.blocks; ++blk, ++uses) {
      // ---- S^T = K Q^T: 16 tokens x 8 head slots, 8 steps of 16 dims
      wait_stage(&H.full[0], uses & 1, nullptr);
      const uint32_t valid = H.valid[0];
      float sc[4] = {0.f, 0.f, 0.f, 0.f}, sd[4] = {0.f, 0.f, 0.f, 0.f};  // even / odd steps
#pragma unroll
      for (int kk = 0; kk < 8; ++kk) {
        // matrices: tokens 0-7 / 8-15 of dims 16kk..+7, then of dims 16kk+8..+15
        uint32_t a[4];
        ldmatrix_x4(a, tile_chunk(const_cast<uint8_t*>(tileK), (lane & 7) + ((lane >> 3) & 1) * 8,
                                  2 * kk + (lane >> 4)));
        mma_bf16((kk & 1) ? sd : sc, a[0], a[1], a[2], a[3], qb[kk][0], qb[kk][1]);
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&H.empty[0]);
#pragma unroll
      for (int i = 0; i < 4; ++i) sc[i] += sd[i];
      // ---- online softmax per q head (column) over tokens gid, gid + 8 of all lanes with this tig
      float x[4];
      x[0] = gid < valid ? sc[0] * b.scale_log2 : -INFINITY;
      x[1] = gid < valid ? sc[1] * b.scale_log2 : -INFINITY;
      x[2] = gid + 8 < valid ? sc[2] * b.scale_log2 : -INFINITY;
      x[3] = gid + 8 < valid ? sc[3] * b.scale_log2 : -INFINITY;
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
      // ---- O^T += V^T P^T: 8 steps of 16 dims, k = the block's 16 tokens
      wait_stage(&H.full[1], uses & 1, nullptr);
#pragma unroll
      for (int m = 0; m < 8; ++m) {
        // matrices: tokens 0-7 of dims 16m / 16m+8, then tokens 8-15 of dims 16m / 16m+8
        uint32_t a[4];
        ldmatrix_x4_trans(a, tile_chunk(const_cast<uint8_t*>(tileV), (lane & 7) + (lane >> 4) * 8,
                                        2 * m + ((lane >> 3) & 1)));
        mma_bf16(o[m], a[0], a[1], a[2], a[3], ph0, ph1);
        mma_bf16(o[m], a[0], a[1], a[2], a[3], pl0, pl1);
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&H.empty[1]);
    }
    // partial of the item: O^T columns of the group's heads, m and l
    float* base = b.partials + static_cast<uint64_t>(item) * kAttnKvHeads * group * kAttnRecord;
#pragma unroll
    for (int e = 0; e < 2; ++e) {
      const uint32_t hcol = 2 * tig + e;
      if (hcol < group) {
        float* dst = base + static_cast<uint64_t>(head * group + hcol) * kAttnRecord;
#pragma unroll
        for (int m = 0; m < 8; ++m) {
          dst[16 * m + gid] = o[m][e];
          dst[16 * m + gid + 8] = o[m][2 + e];
        }
        if (gid == 0) {
          dst[kAttnHeadDim] = mx[e];
          dst[kAttnHeadDim + 1] = lsum[e];
        }
      }
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
