/*
 * anchorkv_b200 -- C ABI of the B200 (sm_100a) packed-KV decode path.
 *
 * Every entry point takes plain device pointers, sizes and a CUDA stream
 * (passed as void*, a cudaStream_t; NULL means the legacy default stream),
 * returns an int status (AKV_OK on success), launches asynchronously on that
 * stream and allocates nothing: the caller owns every buffer, including the
 * split-K workspace.  Apart from the fixed scratch of
 * akv_packed_attention_static (see its declaration), the library keeps no
 * mutable global state, so concurrent calls on different streams are independent.
 *
 * Reference interfaces each entry point replaces are cited by file:line in
 * the reference project (Dev-Sinha13/Dynamic-Quantization, src/anchorkv/).
 *
 * Physical page format (the layout kernels read and write):
 *   - a page is `block` = 16 tokens of K and V for all KV heads of one
 *     (sequence, layer); it lives at a 16-byte aligned byte offset in an arena;
 *   - the page holds `heads` head records back to back, each
 *     akv_record_bytes(head_dim, group, mode) bytes:
 *       [K payload][V payload][K scales][V scales][zero pad to 16 bytes]
 *     payload = 16 rows x head_dim, fp16 / int8 / two's-complement nibbles
 *     with the even element in the low nibble (the reference byte layout).
 *     K payloads are row-major.  V payloads hold the same bytes with their
 *     16-byte units permuted inside each 128-byte line: row-major offset o is
 *     stored at o ^ (key << 4), where, for token row r and row width
 *     w = head_dim * bits / 8, key = r & 6 (w = 128 or 64), (r >> 1) & 2
 *     (w = 32), or t&1 | (t&2) << 1 with t = (r >> 1) & 3 (w = 256).  The
 *     map is its own inverse.  It makes the decode's V fragment loads free
 *     of shared-memory bank conflicts;
 *     scales = fp16, element (row, col) uses scale (row*head_dim+col)/group;
 *   - a page descriptor is an int64:
 *       bits 0-1  mode (AKV_MODE_*; AKV_MODE_SKIP = evicted or not visible)
 *       bits 2-5  valid tokens in the page minus one (0..15)
 *       bits 8-63 byte offset of the page in the arena (16-byte aligned).
 */
#ifndef ANCHORKV_B200_H
#define ANCHORKV_B200_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Host status codes. */
#define AKV_OK 0
#define AKV_ERR_INVALID 1     /* bad argument: null pointer, size, alignment, dtype */
#define AKV_ERR_UNSUPPORTED 2 /* well-formed but unsupported geometry */
#define AKV_ERR_CUDA 3        /* CUDA error when launching */
#define AKV_ERR_SCRATCH 4     /* request larger than akv_packed_attention_static's fixed scratch */

/* Bits a kernel ORs into the optional status word (int32, caller owned; device
 * memory, or mapped pinned host memory from akv_status_alloc so that the host
 * can read it without synchronising).  Kernels set bits with a plain
 * read-OR-write, not an atomic: two different bits raised at the same moment
 * may leave only one of them, but the word is nonzero after any error. */
#define AKV_DEV_BAD_DESCRIPTOR 1 /* descriptor outside the arena or misaligned; page skipped */
#define AKV_DEV_TIMEOUT 2        /* a bounded wait on a bulk copy gave up */

/* Page modes (descriptor bits 0-1). */
#define AKV_MODE_SKIP 0
#define AKV_MODE_INT4 1
#define AKV_MODE_INT8 2
#define AKV_MODE_FP16 3

/* Quantizer semantics: the reference has two, and they are not bitwise equal. */
#define AKV_SEM_TENSOR 0 /* backend.quantize_tensor: fp32 scale divisor, scale 1 for zero groups */
#define AKV_SEM_PAGE 1   /* packed_decode.pack_page: fp16 scale divisor, scale >= 2^-14 */

/* Element types. */
#define AKV_DTYPE_F32 0
#define AKV_DTYPE_F16 1
#define AKV_DTYPE_BF16 2

/* Message for a host status code. */
const char *akv_status_string(int status);

/* ABI version, bumped on any incompatible change. */
int akv_abi_version(void);

/* A status word in mapped pinned host memory (64 bytes, zeroed): kernels get
 * `*dev_ptr`, the host reads `*host_ptr` with no copy or synchronisation (the
 * bits of a kernel are visible once it has finished).  No counterpart in the
 * reference, which raises exceptions from host code only; this is how the
 * Python layer turns device-side errors (AKV_DEV_*) into exceptions on the
 * next call.  Free with akv_status_free. */
int akv_status_alloc(void **host_ptr, void **dev_ptr);
int akv_status_free(void *host_ptr);

/* Bytes of one (page, head) record for a mode (0 for AKV_MODE_SKIP); -1 for an
 * unsupported geometry.  Replaces the byte accounting of QuantizedPage.nbytes
 * (packed_decode.py:28-32), rounded up to 16 bytes. */
int64_t akv_record_bytes(int head_dim, int group, int mode);

/* Quantize a flat tensor of `numel` elements in groups of `group` (zero padded
 * to a whole group) to symmetric INT8 or packed INT4.
 * payload: int8[padded] (bits 8) or uint8[padded/2] (bits 4); scales: fp16[padded/group].
 * Replaces backend.quantize_tensor (backend.py:183-226) with AKV_SEM_TENSOR and
 * the data plane of packed_decode.pack_page (packed_decode.py:48-67) with AKV_SEM_PAGE. */
int akv_quantize(const void *src, int src_dtype, int64_t numel, int64_t group, int bits,
                 int semantics, void *payload, void *scales, void *stream);

/* Dequantize `numel` elements: out = dtype(int * float(scale)).
 * Replaces PackedTensor.dequantize (backend.py:154-180) and QuantizedPage.dense
 * (packed_decode.py:34-45). */
int akv_dequantize(const void *payload, const void *scales, int64_t numel, int64_t group,
                   int bits, void *out, int out_dtype, void *stream);

/* Quantize/pack dense fp16 K and V into page records.  Page p covers source
 * rows (p / blocks_per_row, tokens (p % blocks_per_row)*16 .. +15) of
 * src[outer][head][token][head_dim] (strides in elements, head_dim contiguous);
 * dst_desc[p] gives its mode and offset.  Bit-exact with quantize_tensor
 * (AKV_SEM_TENSOR, group dividing 16*head_dim) or pack_page (AKV_SEM_PAGE).
 * Replaces the per-block quantize_tensor loop of requantize_segment
 * (backend.py:470-483) and PagedLayer's page packing (packed_decode.py:144-174). */
int akv_pack_pages(const void *src_k, const void *src_v, int64_t outer_stride,
                   int64_t head_stride, int64_t blocks_per_row, int64_t n_pages,
                   const int64_t *dst_desc, void *arena, int64_t arena_bytes, int heads,
                   int head_dim, int group, int semantics, int32_t *dev_status, void *stream);

/* Requantize pages in the arena: dequantize src records to fp16 exactly as
 * QuantizedPage.dense does (fp16(int * float(scale)); FP16 records as stored),
 * then pack into dst records with `semantics`: AKV_SEM_PAGE (pack_page) or
 * AKV_SEM_TENSOR (quantize_tensor on fp16 values).  Source and destination
 * records must not overlap.  Replaces PagedLayer.demote (packed_decode.py:164-174)
 * and the per-block dequantize + quantize_tensor loop of
 * DeclarativeKVCache.requantize_segment (backend.py:470-483). */
int akv_repack_pages(const int64_t *src_desc, const int64_t *dst_desc, int64_t n_pages,
                     void *arena, int64_t arena_bytes, int heads, int head_dim, int group,
                     int semantics, int32_t *dev_status, void *stream);

/* Append decode-step tokens of a batch into FP16 pages: for every sequence b,
 * `rows` token rows of src_k/src_v (fp16 [batch][heads][rows][head_dim] with
 * the given strides in elements, head_dim contiguous, 8-byte aligned) are
 * written at page rows first_row .. first_row + rows - 1 of the page named by
 * table[b * table_stride + page], whose valid-token count becomes
 * first_row + rows.  new_desc (nullable): a fresh FP16 page per sequence, whose
 * descriptor is written into the table first and whose other rows are zeroed.
 * first_row + rows <= 16.  Replaces the per-token page writes and the
 * host-to-device publish of PagedLayer.append (packed_decode.py:126-154), for a
 * batch of sequences in one launch. */
int akv_append_rows(const void *src_k, const void *src_v, int64_t src_batch_stride,
                    int64_t src_head_stride, int64_t src_token_stride, int batch, int rows,
                    int first_row, int64_t *table, int64_t table_stride, int page,
                    const int64_t *new_desc, void *arena, int64_t arena_bytes, int heads,
                    int head_dim, int32_t *dev_status, void *stream);

/* Dequantize pages to dense out_k/out_v[heads][n_pages*16][head_dim] of
 * out_dtype (skipped pages read as zeros): AKV_DTYPE_F16 gives
 * fp16(int * float(scale)) as QuantizedPage.dense; AKV_DTYPE_F32 / _BF16 round
 * int * float(scale) once to that type, as PackedTensor.dequantize does.
 * Replaces PagedLayer.dense (packed_decode.py:189-194) and the block
 * dequantisation of DeclarativeKVCache.materialize_segments (backend.py:557-591). */
int akv_unpack_pages(const int64_t *desc, int64_t n_pages, const void *arena,
                     int64_t arena_bytes, int heads, int head_dim, int group, void *out_k,
                     void *out_v, int out_dtype, int32_t *dev_status, void *stream);

/* Bytes of the workspace akv_decode_partials / akv_packed_attention need for
 * this geometry on the current device (-1 for invalid or unsupported arguments).
 * The workspace holds a 256-byte header describing the work decomposition and
 * one partial state (acc[head_dim], m, l) per (warp, item it touched, query
 * head); it is opaque to the caller and needs no initialisation.  Calls that
 * use one workspace must be ordered (one stream, or events between streams).
 * The size is for the decode's finer cut of the work (see `splits` below); a
 * workspace that only holds exactly `splits` pieces per (sequence, KV head)
 * also works, with that decomposition. */
int64_t akv_workspace_bytes(int batch, int q_heads, int kv_heads, int head_dim, int max_blocks,
                            int splits);

/* Paged decode attention, first stage: one query token per sequence over mixed
 * FP16/INT8/INT4 pages, partial states into the workspace.
 *   table: descriptors, sequence b's pages at table[b*table_stride + j], j < blocks(b);
 *   seq_blocks: per-sequence page count (NULL: every sequence has max_blocks);
 *   query: fp16 [batch][q_heads][head_dim] with the given strides (elements);
 *   q head h attends KV head h / (q_heads / kv_heads);
 *   splits: pieces each (sequence, KV head) is cut into at least, where it has
 *   the pages (the reference's split-K count); the decode cuts finer, down to
 *   16 pages a piece, while the device has resident warps to spare (<= 0: as
 *   many pieces as the device has resident warps).  Results do not depend on
 *   it beyond fp32 rounding.  The kernel is persistent and gives every warp one
 *   contiguous range of (sequence, KV head, page) work.
 * Replaces triton_decode._decode_parts (triton_decode.py:35-67). */
int akv_decode_partials(const void *arena, int64_t arena_bytes, const int64_t *table,
                        int64_t table_stride, const int32_t *seq_blocks, int32_t max_blocks,
                        const void *query, int64_t q_batch_stride, int64_t q_head_stride,
                        int32_t batch, int32_t q_heads, int32_t kv_heads, int32_t head_dim,
                        int32_t group, float scale, int32_t splits, void *workspace,
                        int64_t workspace_bytes, int32_t *dev_status, void *stream);

/* Second stage: log-sum-exp merge of the workspace's partial states per
 * (sequence, query head).  out (nullable): fp16 [batch][q_heads][head_dim] with
 * strides (elements); state_out (nullable): fp32 [batch][q_heads][head_dim + 2]
 * merged (acc, m, l), m in base-2 units of the scaled score and acc, l relative
 * to 2^m, for a further merge (e.g. across GPUs).  Empty shares weigh 0; a
 * query with no visible token gets zeros.
 * Replaces triton_decode._merge_parts (triton_decode.py:70-82). */
int akv_merge(const void *workspace, int32_t batch, int32_t q_heads, int32_t head_dim, void *out,
              int64_t out_batch_stride, int64_t out_head_stride, float *state_out,
              int32_t *dev_status, void *stream);

/* Merge n states fp32 [n][batch][q_heads][head_dim + 2] (as akv_merge's
 * state_out writes them, e.g. gathered from n GPUs holding contiguous shards of
 * each sequence) into the fp16 output [batch][q_heads][head_dim].  The same LSE
 * algebra as triton_decode._merge_parts (triton_decode.py:70-82). */
int akv_merge_states(const float *states, int32_t n, int32_t batch, int32_t q_heads,
                     int32_t head_dim, void *out, int64_t out_batch_stride,
                     int64_t out_head_stride, void *stream);

/* Bytes of one rank's exchange buffer for akv_merge_exchange (-1 if invalid):
 * 64-bit words [2][world][splits][batch * q_heads][head_dim + 2], the leading
 * 2 being the epoch parity, each word an fp32 value in its low half and the
 * epoch of the call that wrote it in its high half; splits (part-states per
 * row) is 4 for up to 32 rows, 2 for up to 64, else 1.  world <= 8. */
int64_t akv_exchange_bytes(int32_t world, int32_t batch, int32_t q_heads, int32_t head_dim);

/* Cross-GPU merge over peer memory for one sequence split over `world` GPUs
 * (each rank decoded its page range into `workspace` with akv_decode_partials):
 * one kernel merges this rank's partials per (sequence, query head) into
 * part-states, stores them into every rank's exchange buffer (plain peer
 * stores over NVLink, every 8-byte word tagged with the epoch), waits
 * (bounded, AKV_DEV_TIMEOUT after 2 s) until every rank's parts of the row
 * carry the epoch, and merges them into `out`.
 * Replaces akv_merge + an all-gather + akv_merge_states.
 *   peer_buffers[r]: rank r's exchange buffer as mapped in this process
 *     (akv_ipc_alloc / akv_ipc_open), zeroed before the first call;
 *   epoch: 1 for the first call on these buffers, +1 for each following call,
 *     the same on every rank; after 0xFFFFFFFF it goes on at 2 (any nonzero
 *     value works that alternates in parity and differs from the epoch two
 *     calls before).  Every rank must make the same calls.
 * Calls of even and odd epochs use separate halves of the buffers, so a rank
 * may run one call ahead of a slower peer: it writes epoch e + 1's states into
 * the other half while the peer still reads epoch e's, and it cannot reach
 * epoch e + 2 before every peer has published e + 1 (which each does only
 * after finishing its call e). */
int akv_merge_exchange(const void *workspace, int32_t batch, int32_t q_heads, int32_t head_dim,
                       void *const *peer_buffers, int32_t rank, int32_t world, uint32_t epoch, void *out,
                       int64_t out_batch_stride, int64_t out_head_stride, int32_t *dev_status,
                       void *stream);

/* Device buffers shared between the processes of one node (CUDA IPC).  No
 * counterpart in the reference.  akv_ipc_alloc allocates `bytes` zeroed bytes
 * on the current device and writes its AKV_IPC_HANDLE_BYTES-byte handle;
 * another process maps it with akv_ipc_open and unmaps it with akv_ipc_close;
 * the owner frees it with akv_ipc_free after every mapping is closed. */
#define AKV_IPC_HANDLE_BYTES 64
int akv_ipc_alloc(int64_t bytes, void **ptr, void *handle);
int akv_ipc_open(const void *handle, void **ptr);
int akv_ipc_close(void *ptr);
int akv_ipc_free(void *ptr);

/* akv_decode_partials followed by akv_merge, partials in the caller's workspace
 * (at least akv_workspace_bytes bytes, 16-byte aligned).  Both kernels are
 * launched as programmatic dependents of their predecessor in the stream, so
 * each starts while the previous one finishes (it waits for it before touching
 * memory).  Replaces triton_decode.packed_attention (triton_decode.py:85-104). */
int akv_packed_attention(const void *arena, int64_t arena_bytes, const int64_t *table,
                         int64_t table_stride, const int32_t *seq_blocks, int32_t max_blocks,
                         const void *query, int64_t q_batch_stride, int64_t q_head_stride,
                         int32_t batch, int32_t q_heads, int32_t kv_heads, int32_t head_dim,
                         int32_t group, float scale, int32_t splits, void *out,
                         int64_t out_batch_stride, int64_t out_head_stride, void *workspace,
                         int64_t workspace_bytes, int32_t *dev_status, void *stream);

/* Allocation-free akv_packed_attention.  No counterpart in the reference: it
 * exists for callers that cannot allocate device memory -- hosts that reserve
 * all of HBM for their own pool, latency-critical loops where cudaMalloc/cudaFree
 * would synchronize the device, bindings holding raw pointers but no allocator.
 * The split-K partials live in a fixed array inside the library
 * (akv_static_scratch_bytes() = 8 MiB per GPU, held until process exit), so it
 * allocates nothing.  When the finer cut of the work (see `splits`) needs more,
 * the call runs with exactly `splits` pieces per (sequence, KV head) instead;
 * requests whose partial states exceed 8 MiB even then return AKV_ERR_SCRATCH.
 * The first call on a device looks up the array's device address
 * (cudaGetSymbolAddress) with that device current; make that first call before
 * any stream capture.  The address is kept for the life of the process, so
 * after a cudaDeviceReset of that device (which unloads the library's copy of
 * the array) this entry point must not be called on it again.  Failures of
 * the plan (AKV_ERR_INVALID / AKV_ERR_UNSUPPORTED / AKV_ERR_CUDA) are the ones
 * akv_packed_attention reports.  All calls on a device share the array and it keeps the
 * last call's contents (each call rewrites what it reads, so nothing needs
 * clearing); calls whose kernels overlap on the GPU race on it. */
int akv_packed_attention_static(const void *arena, int64_t arena_bytes, const int64_t *table,
                                int64_t table_stride, const int32_t *seq_blocks, int32_t max_blocks,
                                const void *query, int64_t q_batch_stride, int64_t q_head_stride,
                                int32_t batch, int32_t q_heads, int32_t kv_heads, int32_t head_dim,
                                int32_t group, float scale, int32_t splits, void *out,
                                int64_t out_batch_stride, int64_t out_head_stride,
                                int32_t *dev_status, void *stream);

/* Size in bytes of the fixed scratch akv_packed_attention_static uses (8 MiB). */
int64_t akv_static_scratch_bytes(void);

#ifdef __cplusplus
}
#endif

#endif /* ANCHORKV_B200_H */
