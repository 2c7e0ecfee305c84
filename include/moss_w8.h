/*
 * moss_w8.h - C ABI of the B200 (sm_100a) hot path of the MOSS-Image int8 trainer.
 *
 * The library (moss_image_b200/libmoss_w8.so) exports exactly the functions declared
 * here. Every pointer argument is a raw device (or, where stated, host) address; sizes
 * are element counts; streams are CUDA runtime streams owned by the caller. The library
 * never allocates device memory on behalf of a compute call and never synchronises the
 * host inside one. Work is enqueued on the stream passed in.
 *
 * Return value: 0 (MOSS_OK) on success, otherwise one of the MOSS_ERR_* codes; the
 * calling thread's last message is available from moss_last_error().
 *
 * Device-side failures (a bounded wait that ran out, non-finite weights seen by the
 * quantiser) are reported asynchronously by OR-ing MOSS_STATUS_* bits into the optional
 * `status` word (a device int32 the caller zeroes and reads back when convenient).
 */
#ifndef MOSS_W8_H_
#define MOSS_W8_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#if defined(__GNUC__)
#define MOSS_API __attribute__((visibility("default")))
#else
#define MOSS_API
#endif

struct CUstream_st;
typedef struct CUstream_st* moss_stream_t; /* == cudaStream_t */

/* dtype codes */
#define MOSS_DTYPE_F16 0
#define MOSS_DTYPE_BF16 1
#define MOSS_DTYPE_F32 2

/* return codes */
#define MOSS_OK 0
#define MOSS_ERR_INVALID_ARGUMENT 1
#define MOSS_ERR_UNSUPPORTED 2
#define MOSS_ERR_CUDA 3
#define MOSS_ERR_RING_FULL 4
#define MOSS_ERR_NOT_FOUND 5
#define MOSS_ERR_BUSY 6

/* device status bits */
#define MOSS_STATUS_NONFINITE_WEIGHT 0x1
#define MOSS_STATUS_TIMEOUT_LOAD 0x2
#define MOSS_STATUS_TIMEOUT_MMA 0x4
#define MOSS_STATUS_TIMEOUT_CONVERT 0x8
#define MOSS_STATUS_TIMEOUT_EPILOGUE 0x10
#define MOSS_STATUS_TIMEOUT_DRAIN 0x20

/* Library version (major * 10000 + minor * 100 + patch). */
MOSS_API int moss_version(void);

/* Message of the last failed call on this host thread ("" if none). */
MOSS_API const char* moss_last_error(void);

/*
 * Host-visible copy of the GEMM failure bits, so that a host can notice a failed launch
 * without synchronising the device. The first call on a device (with that device current)
 * allocates one word of mapped, portable pinned host memory for it; later calls return the
 * same word. From then on every GEMM launched on that device that sets MOSS_STATUS_* bits in
 * its `status` word also ORs them into this host word (a plain store over the host link, only
 * on the failure path). The caller reads and clears it through *host_word.
 * New in this library: the reference surfaces no device-side failures
 * (training/quant_kernels.py:294-373 launch Triton kernels without a status channel).
 */
MOSS_API int moss_status_mirror(int** host_word);

/*
 * Test hook for the failure path: the next GEMM call from this host thread, if it runs the
 * operand-swapped (few-row) kernel, makes that kernel's MMA issuer wait on a barrier that
 * nothing arrives on. The wait is bounded (about two seconds), so the kernel then sets
 * MOSS_STATUS_TIMEOUT_MMA, every role leaves its loop, the copies and MMAs in flight are
 * drained, TMEM is freed and the launch returns with a garbage result; the context stays
 * usable. Other kernels ignore the request; it is consumed by the next GEMM call either way.
 * New in this library (no counterpart in the reference).
 */
MOSS_API int moss_debug_stall_next_gemm(void);

/*
 * Per-output-channel symmetric int8 quantiser.
 * Replaces the quantiser in FrozenInt8Linear.__init__ (training/quantization.py:87-91):
 *   s[n] = max_k |float(w[n,k])| / 127 (IEEE f32 division); s[n] = 1 where it is 0;
 *   q[n,k] = clamp(round_half_even(float(w[n,k]) / s[n]), -127, 127).
 * w: device [n, k] row-major in w_dtype (F16/BF16/F32). q: device int8 [n, k]. scale: device
 * f32 [n]. Non-finite input sets MOSS_STATUS_NONFINITE_WEIGHT in *status (if given).
 */
MOSS_API int moss_w8_quantize(const void* w, int w_dtype, int64_t n, int64_t k, int8_t* q, float* scale,
                     int* status, moss_stream_t stream);

/*
 * Decoded weight out[n,k] = round_w(float(q[n,k]) * round_w(scale[n])) in out_dtype.
 * Replaces _dequantize (training/quantization.py:23-24), used by the transient
 * FrozenInt8Linear.weight accessor (training/quantization.py:112-114).
 */
MOSS_API int moss_w8_dequantize(const int8_t* q, const float* scale, int64_t n, int64_t k, int out_dtype,
                       void* out, moss_stream_t stream);

/*
 * Scratch bytes the GEMM entry points use for the given problem (k_red = reduction length,
 * n_out = output columns), 0 when none. Two cases split the reduction across CTAs and
 * exchange f32 partial tiles through this workspace: small-M problems (split-K over every
 * tile), and CTA-pair problems whose 256 x 256 tiles leave the last round of the persistent
 * grid partly empty (only that round's tiles are split, so idle SM pairs share them; at most
 * about 19 MB). With a NULL or smaller workspace they run unsplit: lower occupancy, and a
 * result that can differ in the last bit of some outputs, since the f32 partial sums are
 * grouped differently. Either way the result is deterministic for a given call. New in this
 * library: the reference's Triton launchers take no workspace
 * (training/quant_kernels.py:294-373).
 */
MOSS_API int moss_w8a16_gemm_workspace_bytes(int64_t m, int64_t n_out, int64_t k_red, size_t* bytes);

/*
 * Weight-only int8 GEMM, forward:
 *   y[m, n] = round_x( sum_k x[m,k] * dec(q)[n,k]  + round_x(bias[n])
 *                      + lora_scale * sum_j lora_xa[m,j] * round_x(lora_b[n,j]) )
 * with dec(q)[n,k] = round_x(round_w(q[n,k] * round_w(scale[n]))), f32 accumulation in TMEM.
 * Replaces triton_int8_linear_forward (training/quant_kernels.py:294-334) and its kernel
 * (:100-167); the optional LoRA term fuses the update of LoRALinear.forward
 * (training/lora.py:85-86) into the same accumulator.
 *   x       device [m, k] contiguous, x_dtype F16 or BF16 (the compute dtype)
 *   q/scale device int8 [n, k] / f32 [n]; weight_dtype = the module dtype used for decode
 *   bias    nullable device [n] in bias_dtype
 *   lora_xa nullable device [m, lora_rank] in x_dtype (x @ lora_A^T, unscaled)
 *   lora_b  device [n, lora_rank] in lora_b_dtype (required when lora_xa is given)
 *   y       device [m, n] contiguous in y_dtype
 *   workspace nullable device scratch (256-byte aligned) of moss_w8a16_gemm_workspace_bytes(m, n, k)
 */
MOSS_API int moss_w8a16_gemm_fwd(const void* x, int x_dtype, int64_t m, int64_t k, const int8_t* q,
                        const float* scale, int weight_dtype, int64_t n, const void* bias,
                        int bias_dtype, const void* lora_xa, const void* lora_b, int lora_b_dtype,
                        int64_t lora_rank, float lora_scale, void* y, int y_dtype, void* workspace,
                        size_t workspace_bytes, int* status, moss_stream_t stream);

/* Size of the split-K scratch array compiled into the library for moss_w8a16_gemm_fwd_noalloc. */
#define MOSS_W8A16_NOALLOC_SCRATCH_BYTES ((size_t)4 << 20)

/*
 * The forward GEMM above, for callers that cannot allocate device memory on this path: a
 * host whose HBM belongs to another allocator (a caching pool that has reserved the free
 * memory, where a side cudaMalloc fails or makes the pool give memory back), or an FFI
 * caller (cgo, JNI, ctypes) with no device allocator of its own to pass a workspace from.
 * Same arguments and result as moss_w8a16_gemm_fwd, minus the workspace: the split-K scratch
 * is a fixed MOSS_W8A16_NOALLOC_SCRATCH_BYTES array inside the library (one copy on every
 * device that loads the library, held until the process exits). It calls no cudaMalloc,
 * cudaFree or other allocating routine; the caller still passes x, q, scale, y and status.
 *   - The first call on a device, with that device current, looks up the array's device
 *     address (cudaGetSymbolAddress) and caches it; make that first call before any stream
 *     capture.
 *   - The array's memory is committed when the library's device code is loaded on a device.
 *     Under lazy module loading (CUDA_MODULE_LOADING=LAZY, the default) that is this first
 *     call, or the first launch of any of this library's kernels there, and it can then fail
 *     with an out-of-memory error if another pool has already reserved the free memory. Make
 *     the first call at start-up, before such a pool grows, or set CUDA_MODULE_LOADING=EAGER.
 *   - Small-M problems whose moss_w8a16_gemm_workspace_bytes(m, n, k) exceeds the array are
 *     refused with MOSS_ERR_INVALID_ARGUMENT before any launch; use moss_w8a16_gemm_fwd for
 *     them. CTA-pair problems whose last-round split would not fit run without that split.
 *   - All calls on a device share the one array and it keeps the previous call's contents:
 *     each call clears the split-K counters on its stream, and the partial tiles are written
 *     before they are read. Calls whose kernels can overlap on the GPU (different streams
 *     without an ordering event, or different host threads) race on the array; the caller
 *     must serialise them.
 * No counterpart in the reference: its Triton launchers have no scratch and allocate their
 * outputs through torch.
 */
MOSS_API int moss_w8a16_gemm_fwd_noalloc(const void* x, int x_dtype, int64_t m, int64_t k,
                                const int8_t* q, const float* scale, int weight_dtype, int64_t n,
                                const void* bias, int bias_dtype, const void* lora_xa,
                                const void* lora_b, int lora_b_dtype, int64_t lora_rank,
                                float lora_scale, void* y, int y_dtype, int* status,
                                moss_stream_t stream);

/*
 * Weight-only int8 GEMM, grad-input (no weight gradient: the base is frozen):
 *   dx[m, k] = round_g( sum_n dy[m,n] * dec(q)[n,k]
 *                       + lora_scale * sum_j lora_dyb[m,j] * round_g(lora_a[j,k]) )
 * stored in dx_dtype. The int8 weight is read in its [n, k] storage order; the transpose is
 * expressed in the shared-memory operand layout, never materialised.
 * Replaces triton_int8_linear_backward (training/quant_kernels.py:337-373) and its kernel
 * (:170-228); the LoRA term is the input gradient of LoRALinear's adapter branch
 * (training/lora.py:85-86).
 *   dy       device [m, n] contiguous, dy_dtype F16 or BF16
 *   lora_dyb nullable device [m, lora_rank] in dy_dtype (dy @ lora_B, unscaled)
 *   lora_a   device [lora_rank, k] in lora_a_dtype (required when lora_dyb is given)
 *   workspace nullable device scratch (256-byte aligned) of moss_w8a16_gemm_workspace_bytes(m, k, n)
 */
MOSS_API int moss_w8a16_gemm_dx(const void* dy, int dy_dtype, int64_t m, int64_t n, const int8_t* q,
                       const float* scale, int weight_dtype, int64_t k, const void* lora_dyb,
                       const void* lora_a, int lora_a_dtype, int64_t lora_rank, float lora_scale,
                       void* dx, int dx_dtype, void* workspace, size_t workspace_bytes, int* status,
                       moss_stream_t stream);

/*
 * ConvRot grad-input: dx = H * (dy * dec(q)), i.e. moss_w8a16_gemm_dx (no LoRA term) followed
 * by the grouped Hadamard rotation of moss_hadamard_rotate on each row of dx, with the same
 * roundings (the GEMM output rounded to dx_dtype, then every radix stage). When the CTA-pair
 * kernel runs the GEMM and group is 256, the rotation is applied to the accumulator rows in its
 * epilogue (no second pass over dx); otherwise the rotation kernel runs on dx afterwards, on the
 * same stream. group: a power of two <= 8192 that divides k. Replaces triton_convrot_backward
 * (training/quant_kernels.py:469-504), which runs the GEMM and then one kernel per radix stage.
 */
MOSS_API int moss_w8a16_gemm_dx_rotated(const void* dy, int dy_dtype, int64_t m, int64_t n, const int8_t* q,
                               const float* scale, int weight_dtype, int64_t k, int64_t group, void* dx,
                               int dx_dtype, void* workspace, size_t workspace_bytes, int* status,
                               moss_stream_t stream);

/*
 * Grouped normalised Hadamard rotation of the last dimension (ConvRot), y = x . H with H
 * block-diagonal in `group`-sized blocks (a power of two, at most 8192) built from the
 * regular H4 and one H2 factor for odd log2(group). H is symmetric and orthonormal, so the
 * same call rotates activations forward and input gradients back. Every radix stage is
 * computed in f32 and rounded to the tensor's dtype, as the reference's staged transform does
 * (identical results for every value whose intermediate magnitudes stay in the normal range);
 * all stages run in one pass. Replaces triton_hadamard_transform
 * (training/quant_kernels.py:387-426) and its stage kernels (:231-277); eager equivalent
 * rotate_hadamard (training/convrot.py:36-63).
 *   x, y   device [rows, cols] contiguous in dtype (F16, BF16 or F32); y == x is allowed,
 *          otherwise the two must not overlap; cols % group == 0
 */
MOSS_API int moss_hadamard_rotate(const void* x, int dtype, int64_t rows, int64_t cols, int64_t group, void* y,
                         moss_stream_t stream);

/*
 * Per-sequence conditioning of a packed token stream (replaces the index_select expansion
 * of _modulation_sample_indices/_condition_for_tokens and the elementwise ops that consume
 * it, training/model.py:288-312,752-771). Rows [offsets[s], offsets[s+1]) of the
 * [rows, dim] stream belong to sequence s; its condition is row s of scale/shift/gate,
 * whose rows are cond_stride elements apart (views of a [segments, 6, dim] modulation need
 * no copy). offsets: device int64 [segments + 1], offsets[0] = 0, offsets[segments] = rows.
 * The result dtype is x's when cond has the same dtype, else F32 (torch type promotion);
 * every product and sum is rounded to it in the reference's order (no FMA contraction).
 *   modulate  y = x * (1 + scale[s]) + shift[s]       (1 + scale rounded to cond dtype)
 *   gate      y = x + update * gate[s]                (update has x's dtype)
 * The backward entry points write the gradient of x (modulate) or of update (gate),
 * rounded like the reference's autograd, and, when dscale/dshift/dgate are non-null, ADD
 * the per-sequence condition gradients into those f32 [segments, dim] arrays (summed in f32;
 * the caller zeroes them and rounds to the condition dtype).
 */
MOSS_API int moss_segment_modulate(const void* x, int x_dtype, int64_t rows, int64_t dim, const void* scale,
                          const void* shift, int cond_dtype, int64_t cond_stride, const int64_t* offsets,
                          int64_t segments, void* y, moss_stream_t stream);
MOSS_API int moss_segment_modulate_bwd(const void* dy, const void* x, int x_dtype, int64_t rows, int64_t dim,
                              const void* scale, int cond_dtype, int64_t cond_stride, const int64_t* offsets,
                              int64_t segments, void* dx, float* dscale, float* dshift, moss_stream_t stream);
MOSS_API int moss_segment_gate(const void* x, const void* update, int x_dtype, int64_t rows, int64_t dim,
                      const void* gate, int cond_dtype, int64_t cond_stride, const int64_t* offsets,
                      int64_t segments, void* y, moss_stream_t stream);
MOSS_API int moss_segment_gate_bwd(const void* dy, const void* update, int x_dtype, int64_t rows, int64_t dim,
                          const void* gate, int cond_dtype, int64_t cond_stride, const int64_t* offsets,
                          int64_t segments, void* dupdate, float* dgate, moss_stream_t stream);

/*
 * RMSNorm over the last dimension of x [rows, dim] (contiguous) with the reference's
 * rounding points (RMSNorm.forward, training/model.py:161-172): statistics in f32,
 *   n = round_x(x * rsqrt(mean(x^2) + eps)),   y = round_y(n * w),
 * y's dtype = x's if w has it, else F32. rstd (optional, f32 [rows]) receives the per-row
 * rsqrt for the backward. The backward writes dx (x's dtype) for a frozen w:
 *   dn = round_x(round_y(dy * w)),   dx = round_x(r * dn - x * r^3 * sum(dn * x) / dim).
 * Replaces the per-head q/k norms and the block norms of Block._forward_impl
 * (training/model.py:290,296-297,303).
 */
MOSS_API int moss_rmsnorm_fwd(const void* x, int x_dtype, int64_t rows, int64_t dim, const void* weight, int w_dtype,
                     float eps, void* y, float* rstd, moss_stream_t stream);
MOSS_API int moss_rmsnorm_bwd(const void* dy, const void* x, int x_dtype, int64_t rows, int64_t dim,
                     const void* weight, int w_dtype, const float* rstd, void* dx, moss_stream_t stream);

/*
 * Dense gather of a strided (non-overlapping) view into a contiguous buffer, and the
 * inverse scatter. Used by the activation offload to turn the payload views of
 * _offload_view (training/activation_offload.py:32-61) into one copy-engine transfer and
 * to rebuild the original strides in _restore_layout (training/activation_offload.py:64-77).
 * sizes/strides are host arrays of ndim (<= 8) entries, strides in elements.
 */
MOSS_API int moss_strided_gather(const void* src, int64_t elem_size, int ndim, const int64_t* sizes,
                        const int64_t* strides, void* dst, moss_stream_t stream);
MOSS_API int moss_strided_scatter(const void* src, int64_t elem_size, int ndim, const int64_t* sizes,
                         const int64_t* strides, void* dst, moss_stream_t stream);

/*
 * Pinned-host offload ring (replaces the per-tensor pinned allocation and compute-stream
 * copies of pack/unpack, training/activation_offload.py:116-147).
 * The ring owns one or more cudaHostAlloc segments (grown on demand up to max_bytes and
 * reused across steps) and issues D2H copies on `d2h` and H2D copies on `h2d`, both
 * caller-owned streams, fenced against the compute stream with CUDA events.
 */
MOSS_API int moss_offload_ring_create(int device, size_t segment_bytes, size_t max_bytes, moss_stream_t d2h,
                             moss_stream_t h2d, void** ring);
MOSS_API int moss_offload_ring_destroy(void* ring);
/* Copy nbytes of contiguous device memory at src to the ring once `compute` reaches this
 * point. Returns a ticket. MOSS_ERR_RING_FULL when max_bytes would be exceeded. */
MOSS_API int moss_offload_pack(void* ring, const void* src, size_t nbytes, moss_stream_t compute,
                      int64_t* ticket);
/* Start the H2D copy of a ticket's payload into dst (device, nbytes) on the h2d stream. */
MOSS_API int moss_offload_prefetch(void* ring, int64_t ticket, void* dst);
/* Make `compute` wait until the ticket's H2D copy is complete. */
MOSS_API int moss_offload_wait(void* ring, int64_t ticket, moss_stream_t compute);
/* Drop a ticket; when no ticket is live the ring rewinds to its start. */
MOSS_API int moss_offload_release(void* ring, int64_t ticket);
/* Host address of a ticket's payload (valid until release). */
MOSS_API int moss_offload_host_ptr(void* ring, int64_t ticket, void** host);
/* Counters: bytes packed, bytes restored, live tickets, reserved pinned bytes. */
MOSS_API int moss_offload_stats(void* ring, uint64_t* d2h_bytes, uint64_t* h2d_bytes, int64_t* live,
                       uint64_t* pinned_bytes);
/* Measurement of the copy engines (off by default): with timing on, every later copy gets a
 * pair of CUDA events on its stream. moss_offload_copy_time waits for the timed copies and
 * returns their summed durations and bytes, per direction, since timing was first enabled.
 * New in this library: the reference times nothing (training/activation_offload.py:116-147). */
MOSS_API int moss_offload_set_timing(void* ring, int enable);
MOSS_API int moss_offload_copy_time(void* ring, double* d2h_ms, double* h2d_ms, uint64_t* d2h_timed_bytes,
                           uint64_t* h2d_timed_bytes);

/*
 * Frozen-block stager: the staging-slot state machine of the asynchronous block swap
 * (replaces AsyncBlockStreamer._choose_slot/_stage/_run/_record_*_use/close,
 * training/memory.py:143-255,335-360). Each registered block is one packed pinned-host
 * master (the frozen parameters and buffers of a transformer block, training/memory.py:
 * 442-471); a stage is one H2D copy of a master into a device slot on the caller's copy
 * stream. Slot memory is supplied by the caller with moss_block_stager_set_slot.
 * Events fence the copies: the copy into a slot waits for the last release of that slot,
 * and a lease makes the compute stream wait for the slot's copy.
 */
MOSS_API int moss_block_stager_create(int device, int num_slots, moss_stream_t copy, void** stager);
/* Waits for the copy stream and every slot's last release, then frees the stager.
 * MOSS_ERR_BUSY (nothing freed) while a slot is leased, unless `force` is non-zero. */
MOSS_API int moss_block_stager_destroy(void* stager, int force);
/* Register a pinned host master of nbytes; returns its block id (0, 1, ...). */
MOSS_API int moss_block_stager_add_block(void* stager, const void* host, size_t nbytes, int64_t* block);
/* Give slot `slot` device memory of `capacity` bytes (caller-owned; 256-byte aligned). */
MOSS_API int moss_block_stager_set_slot(void* stager, int slot, void* device, size_t capacity);
/* The slot that holds `block`, else an empty slot, else the first slot neither leased nor
 * holding one of the protected blocks. MOSS_ERR_BUSY if there is none. No state changes. */
MOSS_API int moss_block_stager_select(void* stager, int64_t block, const int64_t* protected_blocks, int n_protected,
                             int* slot);
/* Make `slot` hold `block`: no-op if it already does, otherwise enqueue the H2D copy on the
 * copy stream behind the slot's last release and advance the slot's generation. */
MOSS_API int moss_block_stager_stage(void* stager, int64_t block, int slot, uint64_t* generation);
/* Lease a slot for a block invocation: `compute` waits for the slot's copy.
 * MOSS_ERR_BUSY if the slot is already leased. */
MOSS_API int moss_block_stager_lease(void* stager, int slot, moss_stream_t compute, uint64_t* generation);
/* Keep a leased slot leased past the invocation (a checkpoint recomputation whose block
 * backward has not run yet); its release comes from release(). */
MOSS_API int moss_block_stager_hold(void* stager, int slot);
/* Record the slot's release on `stream` and drop the lease. With block >= 0 the slot must
 * still hold that block at that generation (MOSS_ERR_NOT_FOUND otherwise). */
MOSS_API int moss_block_stager_release(void* stager, int slot, int64_t block, uint64_t generation,
                              moss_stream_t stream);
/* Resident block (-1 if none), generation and lease flag of a slot. */
MOSS_API int moss_block_stager_slot_info(void* stager, int slot, int64_t* block, uint64_t* generation, int* leased);
/* Counters: copies and bytes staged, peak resident blocks; with copy_ms/timed_bytes
 * non-null, waits for the outstanding copies and returns their summed copy-engine time. */
MOSS_API int moss_block_stager_stats(void* stager, uint64_t* copies, uint64_t* bytes, int* peak_resident,
                            double* copy_ms, uint64_t* timed_bytes);

#ifdef __cplusplus
}
#endif

#endif /* MOSS_W8_H_ */
