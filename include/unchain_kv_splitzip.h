/*
 * unchain_kv_splitzip.h -- C ABI of the B200 (sm_100a) splitzip bf16 KV codec.
 *
 * Library: unchainkv_b200/lib/libunchain_kv_splitzip_cuda.so (same file name
 * as the reference build, native/unchain_kv/CMakeLists.txt:21).
 *
 * Conventions shared by every entry point (the reference's,
 * native/unchain_kv/kvq_splitzip_cuda.cu:288-463):
 *   - pointers are device addresses passed as unsigned long long; the caller
 *     owns all memory; `block_ids_ptr` points at int64 block ids on the device
 *     (0 = the contiguous run starting at `block_start`);
 *   - `stream_ptr` is a cudaStream_t (0 = legacy default stream); work is
 *     enqueued asynchronously and nothing is synchronised;
 *   - return > 0: bytes encoded / bytes written; 0: declined (bad argument,
 *     size mismatch, not enough capacity, would not compress); -1: a CUDA
 *     launch failed, message in kvq_splitzip_last_error() as
 *     "<Kernel>: <cudaGetErrorString>" (thread-local);
 *   - codec overflow is reported in band: byte 0 of the stream is 255.
 *
 * Strides and counts are in 16-bit words.  A paged KV layer is the tensor
 * [2, num_blocks, block_size, kv_heads, head_dim] (bf16); plane_stride and
 * block_stride are its strides along dims 0 and 1, block_words the product of
 * dims 2.. .  The packed word order is K plane then V plane, blocks in
 * block-table order -- exactly torch.index_select(kv_layer, 1, ids) flattened.
 */
#ifndef UNCHAIN_KV_SPLITZIP_H_
#define UNCHAIN_KV_SPLITZIP_H_

#ifdef __cplusplus
extern "C" {
#endif

#if defined(__GNUC__)
#define KVQ_API __attribute__((visibility("default")))
#else
#define KVQ_API
#endif

/* Replaces kvq_splitzip_last_error (kvq_splitzip_cuda.cu:288). */
KVQ_API const char* kvq_splitzip_last_error(void);

/* Replaces kvq_splitzip_bf16_encode_mode (kvq_splitzip_cuda.cu:292).
 * fixed6 (bits 6, mode 3) or fixed5 (bits 5, mode 4) encode of `count`
 * contiguous bf16 words.  Needs capacity >= align4(encoded) + 1032 (the
 * reference's scratch rule); the first 36 scratch bytes hold the palette
 * bitmap.  Palette = distinct high bytes in ascending order. */
KVQ_API long long kvq_splitzip_bf16_encode_mode(unsigned long long src_ptr,
                                                unsigned long long dst_ptr,
                                                unsigned long long count,
                                                unsigned long long capacity,
                                                unsigned long long stream_ptr,
                                                int bits);

/* Replaces kvq_splitzip_bf16_encode (kvq_splitzip_cuda.cu:335): bits = 6. */
KVQ_API long long kvq_splitzip_bf16_encode(unsigned long long src_ptr,
                                           unsigned long long dst_ptr,
                                           unsigned long long count,
                                           unsigned long long capacity,
                                           unsigned long long stream_ptr);

/* Replaces kvq_splitzip_bf16_decode_fixed6_blocks (kvq_splitzip_cuda.cu:344).
 * Decode a mode-3 stream and scatter it into the paged cache. */
KVQ_API long long kvq_splitzip_bf16_decode_fixed6_blocks(
    unsigned long long src_ptr, unsigned long long encoded_bytes,
    unsigned long long dst_ptr, unsigned long long count_words,
    unsigned long long block_count, unsigned long long block_words,
    unsigned long long plane_stride, unsigned long long block_stride,
    unsigned long long block_start, unsigned long long block_ids_ptr,
    unsigned long long stream_ptr);

/* Replaces kvq_splitzip_bf16_decode_fixed6 (kvq_splitzip_cuda.cu:370). */
KVQ_API long long kvq_splitzip_bf16_decode_fixed6(
    unsigned long long src_ptr, unsigned long long encoded_bytes,
    unsigned long long dst_ptr, unsigned long long count_words,
    unsigned long long block_count, unsigned long long block_words,
    unsigned long long plane_stride, unsigned long long block_stride,
    unsigned long long block_start, unsigned long long stream_ptr);

/* Replaces kvq_splitzip_bf16_encode_top16 (kvq_splitzip_cuda.cu:381).
 * top16 encode of `count` contiguous words with a 544-byte table
 * ([0,256) K exponent->code, [256,512) V, [512,528) K books, [528,544) V
 * books; code 255 = escape).  Escape entries are written in ascending
 * position order.  Needs capacity >= align4(encoded) + 8, the reference's
 * rule (kvq_splitzip_cuda.cu:390-394), and declines (0) below it: the
 * statistics pass keeps each tile's escape counts inside the stream's own
 * body region until the encode overwrites them, and a last tile of fewer
 * than 47 words keeps its count in the 8 bytes past align4(encoded). */
KVQ_API long long kvq_splitzip_bf16_encode_top16(unsigned long long src_ptr,
                                                 unsigned long long dst_ptr,
                                                 unsigned long long count,
                                                 unsigned long long capacity,
                                                 unsigned long long tables_ptr,
                                                 unsigned long long stream_ptr);

/* Replaces kvq_splitzip_bf16_decode_top16_blocks (kvq_splitzip_cuda.cu:416).
 * Decode a mode-5 stream into the paged cache; escape entries in any order
 * are accepted (sorted streams are patched in registers, others by a
 * device-side fallback pass).  Returns 2*count_words, also when the stream's
 * mode byte is not 5 (then nothing is written), as the reference does. */
KVQ_API long long kvq_splitzip_bf16_decode_top16_blocks(
    unsigned long long src_ptr, unsigned long long encoded_bytes,
    unsigned long long dst_ptr, unsigned long long count_words,
    unsigned long long block_count, unsigned long long block_words,
    unsigned long long plane_stride, unsigned long long block_stride,
    unsigned long long block_start, unsigned long long block_ids_ptr,
    unsigned long long tables_ptr, unsigned long long stream_ptr);

/* Replaces kvq_splitzip_bf16_decode_top16 (kvq_splitzip_cuda.cu:453). */
KVQ_API long long kvq_splitzip_bf16_decode_top16(
    unsigned long long src_ptr, unsigned long long encoded_bytes,
    unsigned long long dst_ptr, unsigned long long count_words,
    unsigned long long block_count, unsigned long long block_words,
    unsigned long long plane_stride, unsigned long long block_stride,
    unsigned long long block_start, unsigned long long tables_ptr,
    unsigned long long stream_ptr);

/* ---- extensions (same conventions) ------------------------------------ */

/* Fused gather + top16 encode: replaces the torch.index_select pack of
 * src/unchain_kv/vllm_connector.py:2854-2866 followed by
 * kvq_splitzip_bf16_encode_top16; output bytes are identical to that pair. */
KVQ_API long long kvq_splitzip_bf16_encode_top16_blocks(
    unsigned long long cache_ptr, unsigned long long plane_stride,
    unsigned long long block_stride, unsigned long long block_words,
    unsigned long long block_ids_ptr, unsigned long long block_start,
    unsigned long long block_count, unsigned long long dst_ptr,
    unsigned long long capacity, unsigned long long tables_ptr,
    unsigned long long stream_ptr);

/* Fused gather + fixed6/fixed5 encode: replaces the same pack followed by
 * kvq_splitzip_bf16_encode_mode (vllm_connector.py:3110-3118, 4592). */
KVQ_API long long kvq_splitzip_bf16_encode_mode_blocks(
    unsigned long long cache_ptr, unsigned long long plane_stride,
    unsigned long long block_stride, unsigned long long block_words,
    unsigned long long block_ids_ptr, unsigned long long block_start,
    unsigned long long block_count, unsigned long long dst_ptr,
    unsigned long long capacity, unsigned long long stream_ptr, int bits);

/* One call of a batch: a layer (or a request's slice of a layer) of the paged
 * cache and its stream buffer.  Encode reads `cache_ptr` through the block
 * table and writes `stream_ptr` (capacity `stream_bytes`); decode reads
 * `stream_bytes` bytes of `stream_ptr` and scatters into `cache_ptr`.
 * `tables_ptr` is the layer's 544-byte top16 table (ignored by fixed6). */
typedef struct kvq_splitzip_job {
  unsigned long long cache_ptr;
  unsigned long long plane_stride;
  unsigned long long block_stride;
  unsigned long long block_words;
  unsigned long long block_ids_ptr;
  unsigned long long block_start;
  unsigned long long block_count;
  unsigned long long stream_ptr;
  unsigned long long stream_bytes;
  unsigned long long tables_ptr;
} kvq_splitzip_job;

/* Batched forms: `count` jobs (host array) in as few launches as possible
 * (up to 96 jobs per launch), so per-layer calls do not each pay a launch
 * and a single wave of CTAs.  Each job follows the rules of its single-call
 * counterpart; if any job would be declined nothing is launched and 0 is
 * returned.  Encode returns the sum of the jobs' encoded sizes, decode the
 * sum of raw bytes written.  Replaces the per-layer loop of
 * kvq_splitzip_bf16_encode_top16 / _decode_top16_blocks calls the connector
 * makes (src/unchain_kv/vllm_connector.py:3104-3118, 5139-5153). */
KVQ_API long long kvq_splitzip_bf16_encode_top16_batch(const kvq_splitzip_job* jobs,
                                                       unsigned long long count,
                                                       unsigned long long stream_ptr);
KVQ_API long long kvq_splitzip_bf16_encode_mode_batch(const kvq_splitzip_job* jobs,
                                                      unsigned long long count,
                                                      unsigned long long stream_ptr, int bits);
KVQ_API long long kvq_splitzip_bf16_decode_top16_batch(const kvq_splitzip_job* jobs,
                                                       unsigned long long count,
                                                       unsigned long long stream_ptr);
KVQ_API long long kvq_splitzip_bf16_decode_fixed6_batch(const kvq_splitzip_job* jobs,
                                                        unsigned long long count,
                                                        unsigned long long stream_ptr);

/* Device-side codec choice: replaces the connector's host fallback chain
 * top16 -> (D2H, mode byte 255) -> fixed6 -> raw mode 6
 * (src/unchain_kv/vllm_connector.py:3104-3118, 4526-4633).  A read-only
 * statistics pass counts top16 escapes and collects the high-byte palette;
 * the encode pass then writes, per job, the stream the reference chain would
 * end with: top16 (mode 5) if the escapes fit, else fixed6 (mode 3) if <= 64
 * high bytes occur, else raw ([6] + words) when stream_bytes >=
 * align16(2n+1) + scratch, else a fixed6 overflow stream (mode 255) for the
 * host to replace with raw.  The stream's length follows from byte 0
 * (5: 5+n+ceil(n/2)+5*ceil(n/200); 3: 65+n+3*ceil(n/4); 6: 2n+1).
 * Scratch: 64 + align16(8*ceil(tiles/32)) + 16*tiles bytes (tiles = ceil(n/16384)) at
 * the 16-byte aligned end of the largest form.  Returns the sum over jobs of
 * the largest form each job may produce. */
KVQ_API long long kvq_splitzip_bf16_encode_auto_batch(const kvq_splitzip_job* jobs,
                                                      unsigned long long count,
                                                      unsigned long long stream_ptr);

/* Decode whichever stream each job holds (mode 5, 3 or 6, read on the
 * device); `stream_bytes` is the bytes available.  A stream shorter than its
 * mode's length, or with another mode byte, leaves its blocks untouched. */
KVQ_API long long kvq_splitzip_bf16_decode_auto_batch(const kvq_splitzip_job* jobs,
                                                      unsigned long long count,
                                                      unsigned long long stream_ptr);

/* ---- GPU-to-GPU stream transport (replaces the D2H -> TCP -> H2D hop of
 * the compressed-layer frames, src/unchain_kv/tcp_data.py:615-652 and
 * native/unchain_kv/kvq_tcp.cc:224-270): the sender's stream buffers are
 * opened by the receiving process over CUDA IPC, and its decode reads the
 * streams from the sender's HBM over NVLink. */

/* cudaMalloc of a stream buffer on the current device (0 on failure). */
KVQ_API unsigned long long kvq_splitzip_ipc_alloc(unsigned long long bytes);
KVQ_API long long kvq_splitzip_ipc_free(unsigned long long ptr);
/* The 64-byte IPC handle of a kvq_splitzip_ipc_alloc buffer; returns 64. */
KVQ_API long long kvq_splitzip_ipc_get_handle(unsigned long long ptr, unsigned char* handle64);
/* Open a handle from another process on the current device (peer access
 * enabled lazily); its address in this process, 0 on failure. */
KVQ_API unsigned long long kvq_splitzip_ipc_open(const unsigned char* handle64);
KVQ_API long long kvq_splitzip_ipc_close(unsigned long long ptr);
/* 1 if the current device can read peer_device's memory directly. */
KVQ_API long long kvq_splitzip_peer_access(long long peer_device);

/* Codec writeback (vllm_connector.py:3460-3563, 3720-3738): per job, the
 * first stream_bytes of stream_ptr are copied over the job's own blocks,
 * the K-plane run [block_start, block_start + block_count) first, then the
 * V-plane run.  Declines (0) unless block_ids_ptr is 0 and block_stride ==
 * block_words (one contiguous run of adjacent blocks), the stream fits the
 * two runs, and it does not overlap them.  Returns the bytes written. */
KVQ_API long long kvq_splitzip_writeback_batch(const kvq_splitzip_job* jobs,
                                               unsigned long long count,
                                               unsigned long long stream_ptr);

/* The reference's torch-op encoder (vllm_connector.py:3204-3366) on the
 * GPU: per job the first of sign/magnitude (mode 2), high-byte palette
 * (mode 0) and nibble planes (mode 1) that is smaller than raw, else raw
 * (mode 6), chosen on the device from the words' high- and low-byte sets.
 * Needs stream_bytes >= align16(1 + 2n) + 416 (the plan follows the
 * largest form).  Returns the sum of 1 + 2n over the jobs; a stream's
 * length follows from its header. */
KVQ_API long long kvq_splitzip_bf16_encode_torchop_batch(const kvq_splitzip_job* jobs,
                                                         unsigned long long count,
                                                         unsigned long long stream_ptr);

/* Decode whichever stream each job holds, in every form the reference's
 * receiver takes (vllm_connector.py:5098-5313): modes 5, 3 and 6 as
 * kvq_splitzip_bf16_decode_auto_batch, plus the torch-op forms 0 (palette),
 * 1 (nibble planes), 2 (sign/magnitude) and 4 (fixed5), for which
 * stream_bytes must be the exact stream length and the receiver's header
 * checks apply (vllm_connector.py:5168-5278).  A stream that fails them
 * leaves its blocks untouched.  Returns the raw bytes of all jobs (2n each),
 * 0 if declined, -1 on a CUDA error. */
KVQ_API long long kvq_splitzip_bf16_decode_any_batch(const kvq_splitzip_job* jobs,
                                                     unsigned long long count,
                                                     unsigned long long stream_ptr);

/* ---- calibration (GPU form of the exponent-histogram trace that the
 * reference's top16 codebooks come from: vllm_connector.py:2871-2904 counts
 * (w >> 7) & 0xFF per plane with torch.bincount, trace.py:27-58 and
 * scripts/extract_llama_top16_codebooks.py:39-40 rank them). */

/* Exponent histograms of a batch of jobs.  Per job, `stream_ptr` points to
 * 2 x 256 uint32 counters (K plane, then V; stream_bytes >= 2048, 4-byte
 * aligned) to which the counts of the job's words are added; `tables_ptr`
 * is not used.  Returns the number of jobs, 0 if declined, -1 on a CUDA
 * error. */
KVQ_API long long kvq_splitzip_bf16_exponent_histogram_batch(const kvq_splitzip_job* jobs,
                                                             unsigned long long count,
                                                             unsigned long long stream_ptr);

/* Top16 device tables of `layers` layers from their histograms
 * (layers x 2 x 256 uint32): per plane the 16 most frequent observed
 * exponents ranked by (-count, exponent), code = rank, written as the
 * 544-byte table the encoders take (layers x 544 bytes at tables_ptr; the
 * layout of splitzip_cuda.py:283-298).  observed_ptr receives layers x 2
 * uint32: the exponents with a nonzero count per plane.  With fewer than
 * 16, the remaining codes take the unobserved exponents in ascending order
 * (the reference's extractor rejects such a layer).  Returns layers, 0 if
 * declined, -1 on a CUDA error. */
KVQ_API long long kvq_splitzip_top16_tables_from_histograms(unsigned long long hist_ptr,
                                                           unsigned long long layers,
                                                           unsigned long long tables_ptr,
                                                           unsigned long long observed_ptr,
                                                           unsigned long long stream_ptr);

/* Count of device-side bounded waits that ran out on the current device
 * since load or the last reset (0 in normal operation).  Synchronous; -1 on
 * CUDA error.  A wait that runs out while a stream is encoded also gives
 * that stream a mode-255 header (no receiver decodes it).  Replaces the
 * reference's unbounded spin (kvq_splitzip_cuda.cu:51-55), which has no
 * status. */
KVQ_API long long kvq_splitzip_device_errors(void);

/* Reset that count to 0 on the current device.  Synchronous; 0, or -1 on
 * CUDA error. */
KVQ_API long long kvq_splitzip_device_errors_reset(void);

/* Test hook of the bounded waits (no counterpart in the reference): the
 * encode of kvq_splitzip_bf16_encode_mode with its statistics pass built
 * with a limit of 4 tries per wait and its producer leaving the full barrier
 * of tile `skip_tile` (16384-word tiles) one arrival short.  That wait runs
 * out: the count above grows, the stream gets a mode-255 header, the call
 * returns like kvq_splitzip_bf16_encode_mode.  Nothing faults or waits
 * without a limit. */
KVQ_API long long kvq_splitzip_test_encode_mode_skip_arrival(unsigned long long src_ptr,
                                                             unsigned long long dst_ptr,
                                                             unsigned long long count,
                                                             unsigned long long capacity,
                                                             unsigned long long stream_ptr, int bits,
                                                             unsigned long long skip_tile);

/* ABI revision of the extension entry points. */
KVQ_API long long kvq_splitzip_abi_version(void);

/* top16 encode that allocates nothing (no counterpart in the reference).
 * Same arguments, capacity rule (align4(encoded) + 8), stream bytes and
 * return values as kvq_splitzip_bf16_encode_top16, for callers that cannot
 * allocate device memory while they encode: serving engines that give nearly
 * all of HBM to their paged KV pool (a transient allocation can fail there)
 * and paths that must not call cudaMalloc / cudaFree (those can synchronise
 * the device).  The escape counts of its statistics pass live in a
 * 133,184-byte static device array of this library, held by every GPU that
 * loads it until exit, so it writes no byte of the caller's buffer past the
 * stream.  count above 2^27 words (134,217,728) returns -1 with a message in
 * kvq_splitzip_last_error().  The first call on a device looks up the
 * array's device address with that device current and keeps it for the
 * process; if the lookup fails, the call returns -1 with the CUDA error in
 * kvq_splitzip_last_error().  A process that resets a device
 * (cudaDeviceReset) must not call this entry point on that device again: the
 * kept address belongs to the old context.  All calls share the array (each
 * clears it first): calls that overlap on the GPU, e.g. on concurrent
 * streams, race. */
KVQ_API long long kvq_splitzip_bf16_encode_top16_noalloc(unsigned long long src_ptr,
                                                         unsigned long long dst_ptr,
                                                         unsigned long long count,
                                                         unsigned long long capacity,
                                                         unsigned long long tables_ptr,
                                                         unsigned long long stream_ptr);

/* ---- codec-aware decode attention (extension) ---------------------------
 * The reference's receiver decodes each transfer stream into its paged cache
 * and runs attention on the bf16 copy (scripts/bench_codec_attention.py:
 * 155-157).  This attends over the streams directly.
 *
 * One request of a decode-attention batch: its transfer stream of one layer
 * (the codec's output for the request's `blocks` paged blocks, K plane then
 * V plane, of shape [16 tokens, 8 kv heads, 128 dims] per block: fixed6
 * mode 3, raw mode 6, or top16 mode 5 with `tables_ptr`, the layer's
 * 544-byte table, and its escape entries sorted by position as this
 * library's encoders write them), the number of valid tokens (the last
 * block may be partial), and its query and output, bf16 [8 * group][128]
 * (q head kv_head * group + i attends with kv head kv_head).  tables_ptr
 * may be 0 for requests that are not top16.  (ABI revision 3 added
 * tables_ptr.) */
typedef struct kvq_splitzip_attn_request {
  unsigned long long stream_ptr;
  unsigned long long stream_bytes;
  unsigned long long blocks;
  unsigned long long ctx_tokens;
  unsigned long long q_ptr;
  unsigned long long out_ptr;
  unsigned long long tables_ptr;
} kvq_splitzip_attn_request;

/* Device workspace bytes kvq_splitzip_attention_decode needs for this batch
 * on the current device (0 if the batch would be declined): the partial
 * results of the kernel's work items and, when a request carries top16
 * tables, the scaled scores of every block (512 x group bytes a block),
 * from which the V escapes' correction is computed. */
KVQ_API long long kvq_splitzip_attention_workspace_bytes(const kvq_splitzip_attn_request* reqs,
                                                         unsigned long long count,
                                                         unsigned long long group);

/* out = softmax(q K^T / sqrt(128)) V for every q head of every request, K
 * and V read from the streams, fp32 accumulation, bf16 output.  group: q
 * heads per kv head, 1..16; count: 1..64 requests.  Returns count, 0 if
 * declined (shape, sizes or workspace too small), -1 on a CUDA error.  A
 * stream whose mode byte is not 3, 6 or (with tables) 5 yields zeros for
 * its request and counts one device error, as do top16 entries found out
 * of order. */
KVQ_API long long kvq_splitzip_attention_decode(const kvq_splitzip_attn_request* reqs, unsigned long long count,
                                                unsigned long long group, unsigned long long workspace_ptr,
                                                unsigned long long workspace_bytes, unsigned long long stream_ptr);

/* Kernel profiler (extension; the device-side analogue of the reference's
 * UNCHAIN_KV_TRACE_CUDA event pairs, src/unchain_kv/vllm_connector.py:
 * 3100-3124).  enable(1) clears the record and brackets every later kernel
 * launch of this library with CUDA events on its stream; collect() waits for
 * the recorded launches and returns the number of distinct kernels; name(i),
 * ms(i) and launches(i) read the per-kernel totals. */
KVQ_API long long kvq_splitzip_profile_enable(int on);
KVQ_API long long kvq_splitzip_profile_collect(void);
KVQ_API const char* kvq_splitzip_profile_name(int i);
KVQ_API double kvq_splitzip_profile_ms(int i);
KVQ_API long long kvq_splitzip_profile_launches(int i);

#ifdef __cplusplus
}
#endif

#endif /* UNCHAIN_KV_SPLITZIP_H_ */
