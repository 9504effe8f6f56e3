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
//   - consumer warp h (kv head h): decodes its head's 16 x 128 slice into a
//     swizzled bf16 tile in shared memory, loads tensor-core fragments with
//     ldmatrix, S = Q K^T on m16n8k16 bf16 MMAs (the g q heads of the group
//     as rows), online softmax in fp32 (base 2), O += P V on MMAs with P
//     kept in registers as two bf16 parts (hi + lo);
//   - the item's partial (m, l, O) per q head goes to a workspace and
//     AttnCombineKernel merges the items of each request.
// The QK/PV tiles have g useful rows (4 for the benchmark), so they run on
// warp-level MMAs (16 rows); the kernel is bound by the HBM read of the
// compressed K/V.
#pragma once

#include "splitzip_kernels.cuh"

namespace ukv {

constexpr int kAttnHeadDim = 128;
constexpr int kAttnBlockTokens = 16;
constexpr int kAttnKvHeads = kWarps;  // one consumer warp per kv head
constexpr uint32_t kAttnBlockWords = kAttnBlockTokens * kAttnKvHeads * kAttnHeadDim;  // per plane
constexpr int kAttnStages = 4;
constexpr uint32_t kAttnStageBytes = 2 * kAttnBlockWords + 64;  // raw words of one plane block + pads
constexpr uint32_t kAttnCodesOffset = kAttnBlockWords + 32;     // fixed6 codes inside a stage
constexpr uint32_t kAttnTileBytes = kAttnBlockTokens * kAttnHeadDim * 2;  // one warp's bf16 tile
// dynamic shared memory: the ring stages, then one tile per consumer warp
constexpr uint32_t kAttnSmemBytes = kAttnStages * kAttnStageBytes + kAttnKvHeads * kAttnTileBytes;
constexpr int kAttnMaxReqs = 64;
constexpr int kAttnMaxItems = 1024;
constexpr int kAttnMaxCtas = 320;
constexpr int kAttnMaxGroup = 16;
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

// A warp's 16-token x 128-dim bf16 tile: rows of 16 chunks of 16 bytes, chunk
// c of row t stored at chunk c ^ (t & 7) (ldmatrix reads 8 rows of one logical
// chunk without bank conflicts).
__device__ __forceinline__ uint8_t* tile_chunk(uint8_t* tile, uint32_t t, uint32_t c) {
  return tile + t * 256 + ((c ^ (t & 7)) << 4);
}

// Decode this warp's head slice of a staged plane block into its tile: 128
// units of 16 words (token t = u / 8, dims 16 * (u % 8)), 4 per lane.
__device__ __forceinline__ void attn_decode_tile(const AttnDesc& d, const uint8_t* stage, const uint8_t* pair,
                                                 uint8_t* tile, int head, int lane) {
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    const uint32_t u = lane + 32 * k;
    const uint32_t t = u >> 3, g = u & 7;
    const uint32_t w0 = t * (kAttnKvHeads * kAttnHeadDim) + head * kAttnHeadDim + 16 * g;  // word in the block
    uint32_t o[8];
    if (d.mode == 3) {
      uint32_t Lw[4];
      smem_read16_window(stage, d.pad_x + w0, Lw);
      uint32_t Q[3];
      smem_read_words<3>(stage + kAttnCodesOffset, d.pad_y + 3 * w0 / 4, Q);
      uint32_t f[8];
      f[0] = (Q[0] << 2) & 0x3FFCu;
      f[1] = (Q[0] >> 10) & 0x3FFCu;
      f[2] = __funnelshift_r(Q[0], Q[1], 22) & 0x3FFCu;
      f[3] = (Q[1] >> 2) & 0x3FFCu;
      f[4] = (Q[1] >> 14) & 0x3FFCu;
      f[5] = __funnelshift_r(Q[1], Q[2], 26) & 0x3FFCu;
      f[6] = (Q[2] >> 6) & 0x3FFCu;
      f[7] = (Q[2] >> 18) & 0x3FFCu;
#pragma unroll
      for (int i = 0; i < 8; ++i)
        o[i] = __byte_perm(Lw[i >> 1], 0, (i & 1) ? 0x4342 : 0x4140) |
               *reinterpret_cast<const uint32_t*>(pair + f[i]);
    } else if (d.mode == 6) {  // raw
      smem_read_words<8>(stage, d.pad_x + 2 * w0, o);
    } else {  // a stream this kernel does not read: zeros (the producer raised an error)
#pragma unroll
      for (int i = 0; i < 8; ++i) o[i] = 0u;
    }
    *reinterpret_cast<uint4*>(tile_chunk(tile, t, 2 * g)) = make_uint4(o[0], o[1], o[2], o[3]);
    *reinterpret_cast<uint4*>(tile_chunk(tile, t, 2 * g + 1)) = make_uint4(o[4], o[5], o[6], o[7]);
  }
}

template <int kMaxR, int kMaxI>
__global__ void __launch_bounds__(kCtaThreads, 1) AttnKernel(const __grid_constant__ AttnBatch<kMaxR, kMaxI> b) {
  extern __shared__ __align__(128) uint8_t ring[];
  __shared__ __align__(16) uint32_t pair[4096];
  __shared__ __align__(16) AttnDesc D[kAttnStages];
  __shared__ AttnRing R;
  const int tid = threadIdx.x;
  const int lane = tid & 31;
  const int warp = tid >> 5;
  ring_init(R);
  __syncthreads();

  if (warp == kProducerWarp) {
    // ------------------------------------------------------------ producer
    // K then V of each block of each item of this CTA; the mode byte and the
    // palette of the item's stream are read once per item
    AttnPos p;
    const uint32_t i_end = blockIdx.x < b.ctas ? b.cta_item[blockIdx.x + 1] : 0u;
    uint32_t item = blockIdx.x < b.ctas ? b.cta_item[blockIdx.x] : 0u;
    for (; item < i_end; ++item) {
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
    producer_acquire(R, p, nullptr);
    if (lane == 0) D[p.s].item = kEndTile;
    producer_commit(R, p);
    return;
  }

  // -------------------------------------------------------------- consumers
  const int head = warp;
  const uint32_t group = b.group;
  const uint32_t row = lane >> 2;     // MMA row = q head of the group (rows >= group are zero)
  const uint32_t quad = lane & 3;
  uint8_t* tile = ring + kAttnStages * kAttnStageBytes + head * kAttnTileBytes;
  int pair_req = -1;
  uint32_t cur = kEndTile;  // current item
  uint32_t qa[8][2];        // Q fragments (a0, a2) per 16-dim step
  float o[16][4];           // O accumulators per 8-dim step (c0, c1 = row; c2, c3 = row + 8, unused)
  float m = -INFINITY, l = 0.f;
  // P of the current block as A fragments, split in two bf16 parts
  // (P = hi + lo, relative error ~2^-16) so that large V values do not
  // amplify the rounding of P
  uint32_t pa0 = 0, pa2 = 0, pb0 = 0, pb2 = 0;

  auto flush = [&]() {
    if (cur == kEndTile) return;
    if (row < group) {
      const uint32_t hq = head * group + row;
      float* dst = b.partials + (static_cast<uint64_t>(cur) * (kAttnKvHeads * group) + hq) * kAttnRecord;
#pragma unroll
      for (int j = 0; j < 16; ++j)
        *reinterpret_cast<float2*>(dst + 8 * j + 2 * quad) = make_float2(o[j][0], o[j][1]);
      if (quad == 0) {
        dst[kAttnHeadDim] = m;
        dst[kAttnHeadDim + 1] = l;
      }
    }
  };

  AttnPos p;
  for (;;) {
    consumer_wait(R, p, nullptr);
    const AttnDesc& d = D[p.s];
    const uint32_t item = d.item;
    if (item == kEndTile) break;
    const int req = static_cast<int>(b.item[item].req);
    if (item != cur) {  // uniform across the consumers
      flush();
      cur = item;
      const uint16_t* qh = b.req[req].q + static_cast<uint64_t>(head * group + row) * kAttnHeadDim;
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        qa[k][0] = row < group ? *reinterpret_cast<const uint32_t*>(qh + 16 * k + 2 * quad) : 0u;
        qa[k][1] = row < group ? *reinterpret_cast<const uint32_t*>(qh + 16 * k + 8 + 2 * quad) : 0u;
      }
#pragma unroll
      for (int j = 0; j < 16; ++j) o[j][0] = o[j][1] = o[j][2] = o[j][3] = 0.f;
      m = -INFINITY;
      l = 0.f;
      if (d.mode == 3 && req != pair_req) {
        consumer_sync();  // every warp is done with the previous table
        for (int i = tid; i < 4096; i += kThreads)
          pair[i] = (static_cast<uint32_t>(d.pal[i & 63]) << 8) | (static_cast<uint32_t>(d.pal[i >> 6]) << 24);
        pair_req = req;
        consumer_sync();
      }
    }
    const uint8_t* stage = ring + p.s * kAttnStageBytes;
    __syncwarp();  // the tile's previous contents were read by every lane
    attn_decode_tile(d, stage, reinterpret_cast<const uint8_t*>(pair), tile, head, lane);
    __syncwarp();
    const uint32_t valid = d.valid;
    if (d.plane == 0) {
      // S = Q K^T over the block's 16 tokens: two n-tiles of 8 tokens
      float s[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
#pragma unroll
      for (int j = 0; j < 2; ++j) {
#pragma unroll
        for (int k = 0; k < 8; k += 2) {
          // matrices: dims 16k, 16k+8, 16(k+1), 16(k+1)+8 of tokens 8j..8j+7
          uint32_t r[4];
          const uint32_t t = 8 * j + (lane & 7);
          ldmatrix_x4(r, tile_chunk(tile, t, 2 * k + (lane >> 3)));
          mma_bf16(s[j], qa[k][0], 0u, qa[k][1], 0u, r[0], r[1]);
          mma_bf16(s[j], qa[k + 1][0], 0u, qa[k + 1][1], 0u, r[2], r[3]);
        }
      }
      // online softmax (base 2) of row `row` over tokens 8j + 2*quad + e
      float x[4];
      float bmax = -INFINITY;
#pragma unroll
      for (int j = 0; j < 2; ++j)
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          const uint32_t tok = 8 * j + 2 * quad + e;
          const float v = tok < valid ? s[j][e] * b.scale_log2 : -INFINITY;
          x[2 * j + e] = v;
          bmax = fmaxf(bmax, v);
        }
      bmax = fmaxf(bmax, __shfl_xor_sync(kFull, bmax, 1));
      bmax = fmaxf(bmax, __shfl_xor_sync(kFull, bmax, 2));
      const float m_new = fmaxf(m, bmax);
      const float alpha = exp2f(m - m_new);  // 0 on the first block (m = -inf)
      float pe[4];
      float bsum = 0.f;
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        pe[i] = exp2f(x[i] - m_new);
        bsum += pe[i];
      }
      bsum += __shfl_xor_sync(kFull, bsum, 1);
      bsum += __shfl_xor_sync(kFull, bsum, 2);
      l = l * alpha + bsum;
      m = m_new;
#pragma unroll
      for (int j = 0; j < 16; ++j) {
        o[j][0] *= alpha;
        o[j][1] *= alpha;
      }
      pa0 = pack_bf16(pe[0], pe[1]);
      pa2 = pack_bf16(pe[2], pe[3]);
      pb0 = pack_bf16(pe[0] - __uint_as_float(pa0 << 16), pe[1] - __uint_as_float(pa0 & 0xFFFF0000u));
      pb2 = pack_bf16(pe[2] - __uint_as_float(pa2 << 16), pe[3] - __uint_as_float(pa2 & 0xFFFF0000u));
    } else {
      // O += P V: 16 n-tiles of 8 dims, k = the block's 16 tokens
#pragma unroll
      for (int j = 0; j < 16; j += 2) {
        // matrices: tokens 0-7 / 8-15 of dims 8j, then of dims 8(j+1)
        uint32_t r[4];
        const uint32_t t = (lane & 7) + ((lane >> 3) & 1) * 8;
        ldmatrix_x4_trans(r, tile_chunk(tile, t, j + (lane >> 4)));
        mma_bf16(o[j], pa0, 0u, pa2, 0u, r[0], r[1]);
        mma_bf16(o[j], pb0, 0u, pb2, 0u, r[0], r[1]);
        mma_bf16(o[j + 1], pa0, 0u, pa2, 0u, r[2], r[3]);
        mma_bf16(o[j + 1], pb0, 0u, pb2, 0u, r[2], r[3]);
      }
    }
    consumer_release(R, p);
    p.next();
  }
  flush();
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
  auto rec = [&](uint32_t i) {
    return b.partials + (static_cast<uint64_t>(Q.first_item + i) * heads + hq) * kAttnRecord;
  };
  float M = -INFINITY;
  for (uint32_t i = lane; i < Q.items; i += 32) M = fmaxf(M, rec(i)[kAttnHeadDim]);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) M = fmaxf(M, __shfl_xor_sync(kFull, M, o));
  float L = 0.f;
  for (uint32_t i = lane; i < Q.items; i += 32) L += exp2f(rec(i)[kAttnHeadDim] - M) * rec(i)[kAttnHeadDim + 1];
  L = warp_sum(L);
  float acc[4] = {0.f, 0.f, 0.f, 0.f};
  for (uint32_t i = 0; i < Q.items; ++i) {
    const float* src = rec(i);
    const float w = exp2f(src[kAttnHeadDim] - M);
    const float4 v = *reinterpret_cast<const float4*>(src + 4 * lane);
    acc[0] += w * v.x;
    acc[1] += w * v.y;
    acc[2] += w * v.z;
    acc[3] += w * v.w;
  }
  const float inv = 1.f / L;
  uint16_t* dst = Q.out + static_cast<uint64_t>(hq) * kAttnHeadDim + 4 * lane;
  *reinterpret_cast<uint2*>(dst) =
      make_uint2(pack_bf16(acc[0] * inv, acc[1] * inv), pack_bf16(acc[2] * inv, acc[3] * inv));
}

}  // namespace ukv
