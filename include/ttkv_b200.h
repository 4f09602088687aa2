/*
 * ttkv_b200.h -- C ABI of libttkv_sm100.so, the B200 (sm_100a) kernels behind the TT-KV
 * compressed-KV attention path.
 *
 * Conventions shared by every entry point:
 *   - plain device pointers, sizes and strides; no allocation inside, no host synchronisation,
 *     no device trap. Scratch memory is passed in by the caller (`workspace`), sized by the
 *     matching *_workspace_bytes function.
 *   - `stream` is a cudaStream_t passed as void*; every launch goes on it.
 *   - return 0 on success, a negative TTKV_ERR_* code on a refusal detected on the host (before
 *     any launch). `ttkv_last_error()` then holds a message for the calling thread.
 *   - problems only visible on the device (a block index outside the cache, a sequence longer
 *     than its block-table row, a decoder index outside the pool) are recorded in `status`
 *     (device int32, TTKV_STATUS_*; first error wins) and the affected request is skipped. The
 *     caller reads `status` when it chooses (once per step), so no launch drains the queue.
 *   - a layer's slot geometry is described by ttkv_layout_t, built by ttkv_layout_init.
 *
 * The byte format is the reference's packed slot format (codec/ttkv_packed_cache.py laid out by
 * vllm_ttkv/layout.py): per token, [K slot][V slot], K slot = [r1 int8 coefficients][fp16 ruler]
 * [H x (d/8 bitmap, ceil(res_k*res_bits/8) MSB-first codes, fp16 ruler)] padded to 16 B, V slot =
 * [H x (bitmap, codes, ruler)] padded to 16 B.
 */
#ifndef TTKV_B200_H
#define TTKV_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define TTKV_ABI_VERSION 5

/* host-side refusals (return values) */
#define TTKV_OK 0
#define TTKV_ERR_ARG (-1)          /* a null pointer, a negative size, an inconsistent shape */
#define TTKV_ERR_LAYOUT (-2)       /* geometry the format cannot express */
#define TTKV_ERR_UNSUPPORTED (-3)  /* valid format, but outside what these kernels implement */
#define TTKV_ERR_ALIGN (-4)        /* a pointer or stride breaks an alignment the kernel needs */
#define TTKV_ERR_WORKSPACE (-5)    /* workspace missing or smaller than *_workspace_bytes */
#define TTKV_ERR_CUDA (-6)         /* a CUDA launch or attribute call failed */

/* device-side status codes (written to `status`) */
#define TTKV_STATUS_OK 0
#define TTKV_STATUS_BLOCK_RANGE 1  /* a block id inside the used prefix is < 0 or >= n_blocks */
#define TTKV_STATUS_ROW_SHORT 2    /* seq_len needs more blocks than the block-table row holds */
#define TTKV_STATUS_DECODER 3      /* a decoder index outside [0, n_decoders) */
#define TTKV_STATUS_SLOT_RANGE 4   /* a slot id < 0 (PAD_SLOT_ID) or >= n_slots on a write */
#define TTKV_STATUS_QUERY 5        /* q_len > seq_len, or a query range outside the batch */
#define TTKV_STATUS_TIMEOUT 6      /* a bounded wait on the tensor-core pipeline ran out */
#define TTKV_STATUS_SEQ_BOUND 7    /* a seq_len above the call's max_seq_len (the read's bound) */

/* element types */
#define TTKV_F32 0
#define TTKV_F16 1
#define TTKV_BF16 2

/* Slot geometry of one layer. Fields up to `align` are inputs; the rest are derived.
 * Replaces vllm_ttkv/layout.py:56-157 (TTKLayout) for the device side. */
typedef struct ttkv_layout {
    int32_t H, d, r1, qbits, res_k, res_bits, v_lanes, v_bits, align;
    int32_t coeff_bytes;   /* r1*qbits/8                                   layout.py:99-105 */
    int32_t k_row_bytes;   /* d/8 + ceil(res_k*res_bits/8) + 2             layout.py:108-110 */
    int32_t v_row_bytes;   /* d/8 + ceil(v_lanes*v_bits/8) + 2             layout.py:112-113 */
    int32_t k_slot_bytes;  /* align_up(coeff + 2 + H*k_row, align)         layout.py:138-141 */
    int32_t v_slot_bytes;  /* align_up(H*v_row, align)                     layout.py:144-145 */
    int32_t v_offset;      /* == k_slot_bytes                               layout.py:122-135 */
    int32_t blob_bytes;    /* k_slot + v_slot                               layout.py:151-153 */
} ttkv_layout_t;

/* Fill the derived fields and validate. Replaces TTKLayout.__post_init__ and its properties
 * (vllm_ttkv/layout.py:84-157), including its refusals (d % 8, res_k > d, v_lanes > d,
 * r1*qbits % 8). */
int ttkv_layout_init(ttkv_layout_t* lay, int32_t H, int32_t d, int32_t r1, int32_t qbits,
                     int32_t res_k, int32_t res_bits, int32_t v_lanes, int32_t v_bits,
                     int32_t align);

/* Message for the last refusal on the calling thread ("" if none). */
const char* ttkv_last_error(void);

/* TTKV_ABI_VERSION of the loaded library. */
int32_t ttkv_abi_version(void);

/* A paged cache region of one layer, viewed as bytes: slot s starts at base + s*row_bytes and
 * row_bytes >= blob_bytes (vLLM rounds a page up to whole model-dtype elements,
 * vllm_ttkv/decode.py:125-157). Slot id = block*block_size + offset (vLLM's flat indexing). */
typedef struct ttkv_cache {
    uint8_t* base;
    int64_t n_slots;
    int64_t row_bytes;
    int32_t block_size;
    int32_t flags;         /* TTKV_CACHE_*; 0 keeps the reference's refusals */
} ttkv_cache_t;

/* Writes skip a token whose slot id is negative (vLLM's PAD_SLOT_ID, which an engine gives the
 * padding tokens of a batch padded to a captured CUDA graph's size) instead of refusing it with
 * TTKV_STATUS_SLOT_RANGE. Slots at or past n_slots are still refused. Without the flag a negative
 * slot is refused, as the reference's write refuses PAD_SLOT_ID (vllm_ttkv/impl.py:217-238). */
#define TTKV_CACHE_SKIP_PAD 1

/* The batch's paging and decoders. Request r owns block_table[r*bt_stride + 0..], its first
 * seq_lens[r] tokens are stored (position = index), and its decoder is
 * decoders[dec_index[r]*dec_stride .. +r1*H*d] (fp32 [r1, H*d], column m = h*d + j, the
 * reference's decoder_f, vllm_ttkv/encode.py:178-211).
 * Optional (null: the decode converts the decoders itself): dec_image, the same decoders as
 * ttkv_decoder_image wrote them, decoder i at dec_image + i*image_stride bytes, and dec_scales
 * [n_decoders * H] from the same call. */
typedef struct ttkv_batch {
    const int32_t* block_table;
    int64_t bt_stride;
    int32_t bt_cols;
    const int32_t* seq_lens;
    int32_t n_reqs;
    const float* decoders;
    int64_t dec_stride;
    const int32_t* dec_index;
    int32_t n_decoders;
    const void* dec_image;
    int64_t image_stride;
    const float* dec_scales;
} ttkv_batch_t;

/* ---------------------------------------------------------------- decoder images
 * No counterpart in the reference: an addition of this library.
 * A decoder is fixed for the life of its request, so the operand form the tensor-core decode
 * stages from it can be made once: per KV head h, the head's [r1, d] slice scaled by 2^-e (the
 * power of two that brings its largest |value| into [2^13, 2^14)) and split into fp16 hi + lo,
 * in the byte layout of the decode's shared-memory operand; and 2^e. A decode given the image
 * stages it with one bulk copy instead of reading and converting the fp32 decoder.
 *   ttkv_decoder_image_bytes: bytes per decoder (H heads), 0 when the tensor-core decode does not
 *     serve the layout (then a decode ignores images);
 *   ttkv_decoder_image: decoders [n, r1, H*d] fp32 (decoder i at decoders + i*dec_stride) ->
 *     image + i*image_stride (16-byte aligned, image_stride >= ttkv_decoder_image_bytes) and
 *     scales[i*H + h]. */
size_t ttkv_decoder_image_bytes(const ttkv_layout_t* lay);
int ttkv_decoder_image(const ttkv_layout_t* lay, const float* decoders, int64_t dec_stride, int32_t n,
                       void* image, int64_t image_stride, float* scales, void* stream);

/* The model's RoPE table in vLLM's layout: [rows, d] = cat(cos, sin) in the model dtype
 * (vllm_ttkv/decode.py:54-122). */
typedef struct ttkv_rope {
    const void* table;
    int32_t dtype;
    int64_t rows;
} ttkv_rope_t;

/* ---------------------------------------------------------------- read: decode
 * One launch per layer for every decode request of the batch (one query token each).
 * Replaces, for all requests at once, vllm_ttkv/impl.py:511-540 (_decode_one: gather, split,
 * cos/sin, krt_from_slots krt_triton.py:320-371, softmax, v_out_from_slots
 * v_out_triton.py:121-155) and the per-request loop around it (impl.py:468-493).
 *   q:    request r's post-RoPE query at q + r*q_stride elements, [HQ, d] contiguous.
 *   out:  request r's output at out + r*out_stride elements, [HQ, d]; only query heads of the
 *         KV heads [head_lo, head_hi) are written (G = HQ/H per KV head).
 *   scale: softmax scale (the model's, e.g. d^-0.5).
 *   max_seq_len: an upper bound of the batch's seq_lens, read only on the host (it sizes the
 *         workspace and is checked against the RoPE table). The launch reads nothing from the
 *         host that varies with the batch, and its grid does not depend on seq_lens, so a stream
 *         capture made with a bound replays any batch of the same request count within it. A
 *         request longer than the bound is refused on the device (TTKV_STATUS_SEQ_BOUND).
 */
size_t ttkv_decode_workspace_bytes(const ttkv_layout_t* lay, int32_t n_reqs, int32_t HQ,
                                   int32_t max_seq_len, int32_t head_lo, int32_t head_hi);
int ttkv_decode_paged(const ttkv_layout_t* lay, const ttkv_cache_t* cache,
                      const ttkv_batch_t* batch, const ttkv_rope_t* rope,
                      const void* q, int32_t q_dtype, int64_t q_stride, int32_t HQ,
                      float scale, int32_t head_lo, int32_t head_hi,
                      void* out, int32_t out_dtype, int64_t out_stride,
                      int32_t max_seq_len, void* workspace, size_t workspace_bytes,
                      int32_t* status, void* stream);

/* ---------------------------------------------------------------- decode, allocation-free
 * No counterpart in the reference: an addition of this library.
 * The same decode as ttkv_decode_paged for callers that cannot hand the library scratch memory:
 * hosts that reach it only through this C ABI and have no device allocator of their own (a C or
 * C++ runtime, an FFI binding without torch), and engines that fix their device-memory budget up
 * front (vLLM sizes its KV cache from the memory left after a profiling pass, so memory taken
 * outside its pool mid-serving can push a later allocation out of memory). The split-K partials
 * go to a static device array of TTKV_NOALLOC_SCRATCH_BYTES that every GPU loading the library
 * holds until the process exits; the call allocates nothing.
 *   - a decode needing more scratch than that (ttkv_decode_workspace_bytes) is refused with
 *     TTKV_ERR_WORKSPACE before any launch;
 *   - the first call on a device looks up that device's copy of the array (once, with the
 *     calling thread's current device); make that first call before any stream capture;
 *   - every call on a device shares the one array and it keeps the last call's contents (every
 *     byte a launch reads it has written first, so nothing is cleared); calls that can overlap
 *     on the GPU (two streams, two threads) race on it, so the caller serialises them;
 *   - the refusal is conservative: the scratch is sized as ttkv_decode_workspace_bytes at the
 *     cache's block size (the larger of the two decode plans), and the argument checks of
 *     ttkv_decode_paged come first;
 *   - the device address of the array is looked up once per device and kept: a device reset
 *     (cudaDeviceReset, or a primary-context reset) invalidates it, so a process that resets a
 *     device must not call this entry point on that device afterwards. */
#define TTKV_NOALLOC_SCRATCH_BYTES (4u * 1024u * 1024u)
int ttkv_decode_paged_noalloc(const ttkv_layout_t* lay, const ttkv_cache_t* cache,
                              const ttkv_batch_t* batch, const ttkv_rope_t* rope,
                              const void* q, int32_t q_dtype, int64_t q_stride, int32_t HQ,
                              float scale, int32_t head_lo, int32_t head_hi,
                              void* out, int32_t out_dtype, int64_t out_stride,
                              int32_t max_seq_len, int32_t* status, void* stream);

/* ---------------------------------------------------------------- decode, head-sharded, gathered over NVLink
 * No counterpart in the reference (it has no multi-GPU path): the all-gather of a KV-head-sharded
 * decode's outputs, fused into the decode's segment merge. Every rank of a group of `world`
 * processes (one per GPU) reads its KV heads [head_lo, head_hi) and holds the layer's whole output
 * [n_reqs, HQ, d]; the merge stores each output row into its own `out` AND, at the same byte
 * offset, into every other rank's (peer stores over NVLink); each merge CTA then counts itself on
 * a local ticket word (a GPU-scope release), and the launch's last CTA posts one arrival per merge
 * CTA of the launch to every rank's signal word (system-scope releases, one per rank). ttkv_peer_wait then waits until the local signal word has
 * seen every rank's arrivals for this step, after which `out` holds every head. What it replaces:
 * the copy of a rank's heads into a send buffer, the NCCL all-gather and the copy back.
 *   - out[p] is rank p's `out` pointer (the same view: base, head offset, stride and dtype on every
 *     rank) mapped into this process (ttkv_ipc_open), out[rank] == the `out` argument;
 *   - signal[p] is rank p's signal word for this layer (8 bytes, zeroed once, never reset),
 *     mapped likewise; epoch is this rank's own word for the same layer (local, zeroed once): the
 *     arrivals its waits have taken so far. ttkv_peer_wait adds the step's arrivals to it and
 *     waits until the signal word reaches the sum (so batch sizes may change from step to step);
 *   - a step's arrivals = world * G * (head_hi - head_lo) * n_reqs (every rank's merge CTAs; every
 *     rank runs the same requests);
 *   - served by the tensor-core decode only; other layouts are refused (TTKV_ERR_UNSUPPORTED) and
 *     the caller gathers another way. world <= TTKV_MAX_PEERS.
 * The wait is bounded (about 2 s): a rank that never arrives sets TTKV_STATUS_TIMEOUT; the count
 * waited for still advances, and the group is then out of step and must be rebuilt. */
#define TTKV_MAX_PEERS 8
typedef struct {
    int32_t world, rank;
    void* out[TTKV_MAX_PEERS];
    unsigned long long* signal[TTKV_MAX_PEERS];
    unsigned long long* epoch;
    unsigned long long* ticket;   /* this rank's own word for the layer (local, zeroed once): its
                                     merge CTAs count themselves here, and the last of each launch
                                     posts the launch's arrivals to every rank's signal word and
                                     sets it back to zero */
} ttkv_peers_t;
int ttkv_decode_paged_gather(const ttkv_layout_t* lay, const ttkv_cache_t* cache,
                             const ttkv_batch_t* batch, const ttkv_rope_t* rope,
                             const void* q, int32_t q_dtype, int64_t q_stride, int32_t HQ,
                             float scale, int32_t head_lo, int32_t head_hi,
                             void* out, int32_t out_dtype, int64_t out_stride,
                             int32_t max_seq_len, void* workspace, size_t workspace_bytes,
                             const ttkv_peers_t* peers, int32_t* status, void* stream);
int ttkv_peer_wait(const ttkv_peers_t* peers, int64_t arrivals, int32_t* status, void* stream);

/* Device memory shared between the processes of a group through CUDA IPC handles (plain peer
 * mappings, no multicast object): ttkv_ipc_alloc allocates `bytes` (zeroed, on the current
 * device) and writes its handle (ttkv_ipc_handle_bytes bytes) for the other processes, which map
 * it with ttkv_ipc_open and unmap it with ttkv_ipc_close; the owner frees it with ttkv_ipc_free
 * after every peer has closed it. */
size_t ttkv_ipc_handle_bytes(void);
int ttkv_ipc_alloc(size_t bytes, void** ptr, void* handle);
int ttkv_ipc_open(const void* handle, void** ptr);
int ttkv_ipc_close(void* ptr);
int ttkv_ipc_free(void* ptr);

/* ---------------------------------------------------------------- read: continuation
 * Multi-query read for chunked-prefill / prefix-cache continuations: request r has q_len[r]
 * query tokens at q + (q_start[r] + j)*q_stride, [HQ, d] each, at absolute positions
 * seq_len - q_len + j, attending causally to stored rows 0 .. seq_len - q_len + j.
 * Replaces vllm_ttkv/impl.py:725-778 (_prefill_continuation: krt_multi_from_slots
 * krt_triton.py:269-317, softmax, v_out_multi_from_slots v_out_triton.py:249-294), without
 * materialising the [HQ, Q, n] scores. Outputs at out + (q_start[r] + j)*out_stride.
 * With the decoders' operand images (batch->dec_image), 16-bit queries, r1 <= 126 and 16-byte
 * aligned slot rows, one CTA per (request, KV head, block of 128 (query, head) rows) rebuilds
 * each stored tile once and runs the scores and the V readout on the tensor cores; it needs no
 * workspace. Otherwise, for a layout the tensor-core decode serves, the chunks run on it: a
 * request's (query, query head) rows, query-major, in blocks of 8, each block one decode request
 * with a causal limit per row. ttkv_prefill_workspace_bytes sizes the workspace for that plan
 * with caches of 16 tokens per block (for smaller blocks a workspace below the plan's needs makes
 * the call use the fp32 kernel instead). */
size_t ttkv_prefill_workspace_bytes(const ttkv_layout_t* lay, int32_t n_reqs, int32_t HQ,
                                    int32_t max_q_len, int32_t max_seq_len,
                                    int32_t head_lo, int32_t head_hi);
int ttkv_prefill_cont_paged(const ttkv_layout_t* lay, const ttkv_cache_t* cache,
                            const ttkv_batch_t* batch, const ttkv_rope_t* rope,
                            const int32_t* q_start, const int32_t* q_len,
                            const void* q, int32_t q_dtype, int64_t q_stride, int32_t HQ,
                            float scale, int32_t head_lo, int32_t head_hi,
                            void* out, int32_t out_dtype, int64_t out_stride,
                            int32_t max_q_len, int32_t max_seq_len,
                            void* workspace, size_t workspace_bytes,
                            int32_t* status, void* stream);

/* ---------------------------------------------------------------- write
 * Encode n_tok tokens of one layer straight into their slots (slot_mapping[t]).
 * For token t (raw pre-RoPE K and V at k + t*k_stride, v + t*v_stride, [H, d] each):
 *   coefficients -- if `pinvs` is non-null: c = M @ pinv with M the token's [H*d] K row
 *     (m = h*d + j) and pinvs[tok_dec[t]*pinv_stride ..] holding pinv TRANSPOSED, [r1, H*d]
 *     fp32; then the per-token int8 quantisation (vllm_ttkv/encode.py:301-351,
 *     encode_frozen). Otherwise the caller's codes `coeff_q` [n_tok, r1] int8 and rulers
 *     `coeff_scale` [n_tok] fp32 (the fit path, codec/ttkv_packed_cache.py:353-356) are used;
 *   residual -- R = K - (cq*cs) @ decoder (decoders[tok_dec[t]*dec_stride ..], [r1, H*d] fp32),
 *     top-res_k lanes per head row, quantised and packed;
 *   V        -- top-v_lanes per head row, quantised and packed.
 * Byte-identical to the reference's fused writer (vllm_ttkv/encode.py:511-579 _fused_write,
 * select_triton.py:157-232) given the same fp32 coefficients and residual; ties in magnitude
 * keep the lowest lane. Replaces encode_frozen(_batch) + _fused_write for a whole layer in one
 * launch instead of ~20 launches per request: on the frozen path a cluster of H CTAs per token
 * (one per KV head) projects, reduces the coefficients over the cluster's shared memory,
 * quantises and packs; when the pools' [r1, 128] slices do not fit shared memory (r1 > 200) or
 * are not 16-byte aligned with the pool stride r1*H*d, a projection launch and a pack launch do
 * the same. The frozen path needs ttkv_write_workspace_bytes(lay, n_tok) bytes of workspace
 * (the projected coefficients of the two-launch form). */
size_t ttkv_write_workspace_bytes(const ttkv_layout_t* lay, int32_t n_tok);
int ttkv_write_paged(const ttkv_layout_t* lay, const ttkv_cache_t* cache,
                     const int64_t* slot_mapping, int32_t n_tok,
                     const void* k, int32_t k_dtype, int64_t k_stride,
                     const void* v, int32_t v_dtype, int64_t v_stride,
                     const int32_t* tok_dec, const float* decoders, int64_t dec_stride,
                     const float* pinvs, int64_t pinv_stride, int32_t n_decoders,
                     const int8_t* coeff_q, const float* coeff_scale,
                     void* workspace, size_t workspace_bytes,
                     int32_t* status, void* stream);

/* ---------------------------------------------------------------- write, storage-sharded
 * No counterpart in the reference (it has no multi-GPU path): an addition of this library.
 * The storage-sharded slot format for KV-head tensor parallelism: a GPU holding KV heads
 * [h_lo, h_hi) stores per token the blob of the layout with H' = h_hi - h_lo heads and the same
 * widths: [coefficient block + ruler][its heads' K rows] padded to 16 B, [its heads' V rows]
 * padded to 16 B. Reassembled (coefficient block from any shard, head rows in head order, zero
 * padding) the shards are byte-identical to the full blob ttkv_write_paged writes.
 * `lay` is the FULL layout: k/v, the decoders and the pinv pool cover all H heads, because the
 * coefficients project every head's K (c = M @ pinv); only heads [h_lo, h_hi) are packed, into
 * `cache`, whose rows have the held heads' layout (ttkv_layout_init with H' heads).
 * A read of a shard is ttkv_decode_paged with that layout, the decoders' columns of the held
 * heads ([r1, H'*d] per decoder) and the held heads' query rows.
 * ttkv_write_paged(lay, ...) is ttkv_write_paged_shard(lay, 0, lay->H, ...). */
int ttkv_write_paged_shard(const ttkv_layout_t* lay, int32_t h_lo, int32_t h_hi,
                           const ttkv_cache_t* cache, const int64_t* slot_mapping, int32_t n_tok,
                           const void* k, int32_t k_dtype, int64_t k_stride,
                           const void* v, int32_t v_dtype, int64_t v_stride,
                           const int32_t* tok_dec, const float* decoders, int64_t dec_stride,
                           const float* pinvs, int64_t pinv_stride, int32_t n_decoders,
                           const int8_t* coeff_q, const float* coeff_scale,
                           void* workspace, size_t workspace_bytes, int32_t* status, void* stream);

/* Lane select + quantise + bit-pack of `rows` (head, token)-ordered rows x [rows, d] into the
 * slots: row i = h*n_tok + t lands at slots[t], field_off + h*row_stride. The standalone form
 * of vllm_ttkv/select_triton.py:235-290 (write_rows; write_k_residual / write_v_rows). */
int ttkv_select_pack_rows(const ttkv_cache_t* cache, const int64_t* slots, int32_t n_tok,
                          const void* x, int32_t x_dtype, int32_t heads, int32_t d,
                          int32_t field_off, int32_t row_stride, int32_t lanes, int32_t bits,
                          int32_t* status, void* stream);

/* ---------------------------------------------------------------- fit tail
 * Everything in codec/ttkv_packed_cache.py:337-375 (build_k_layer) after the two SVDs, plus the
 * zero padding of vllm_ttkv/encode.py:287-296:
 *   G1 [n, r] (the token core), G2 [r, d, r2], G3 [r2, H] (fp32, from the TT-SVD, r <= budget)
 *   -> coeff_q [n, budget] int8 (zero past r), coeff_scale [n] fp32 (kept fp32 for the residual;
 *      the slot stores fp16), dec_q [r, H*d] int8, dec_scale [r] fp16 bits,
 *      decoder [budget, H*d] fp32 = dec_q*dec_scale (zero rows past r).
 * `scratch` holds r*H*d + r*d*r2 + r2*H floats. */
size_t ttkv_fit_tail_scratch_bytes(int32_t r, int32_t r2, int32_t H, int32_t d);
int ttkv_fit_tail(const float* G1, const float* G2, const float* G3, int32_t n, int32_t r,
                  int32_t r2, int32_t H, int32_t d, int32_t qbits, int32_t budget,
                  int8_t* coeff_q, float* coeff_scale, int8_t* dec_q, uint16_t* dec_scale,
                  float* decoder, void* scratch, size_t scratch_bytes, void* stream);

#ifdef __cplusplus
}
#endif
#endif /* TTKV_B200_H */
