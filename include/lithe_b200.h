/*
 * lithe_b200.h -- C ABI of the B200 (sm_100a) index-resident multi-adapter LoRA path.
 *
 * Every pointer named "device" is a CUDA device pointer on the current device; every
 * "stream" is a cudaStream_t passed as void*.  No entry point allocates device memory,
 * synchronises the host or keeps a pointer after it returns: the caller owns all buffers
 * and the work is ordered on the given stream only.  Return value: LITHE_OK (0) or a
 * negative LITHE_ERR_* code; lithe_last_error() gives a message for the calling thread.
 *
 * Data formats (identical to the reference implementation, JianJiang1995/LITHE):
 *   - codebook: 512 codewords of 64 values, c_k[t] = (2*popc((k ^ P(t)) & 511) - 9) / 3
 *     with P(t) bit q = parity(t & q), q < 9 (lithe/codebook.py:35-69).  A level-l pool of
 *     side A/B is sigma_l * c_k, so each pool level holds exactly 10 distinct fp32 values
 *     lut[side][l][n] = pool[l][k][t] for n = popc((k ^ P(t)) & 511).  The entry points
 *     take those 10 values per (side, level) instead of the (L,512,64) pools.
 *   - packed index stream (lithe/kernels/packed.py:1-17,38-52): one adapter's indices in
 *     (block, level)-major order, 7 nine-bit indices per little-endian uint64 word; index p
 *     lives in word p/7, bits [9*(p%7), 9*(p%7)+9).  Per module the A blocks come first,
 *     then the B blocks (packed.py:125-133).
 *   - level-major integer banks (lithe/serve.py:58-67, lithe/kernels/layers.py:105-106):
 *     (n_slots, L, n_blocks) int16 or int32.
 */
#ifndef LITHE_B200_H
#define LITHE_B200_H

#include <stdint.h>

#if defined(__GNUC__)
#define LITHE_API __attribute__((visibility("default")))
#else
#define LITHE_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

#define LITHE_OK 0
#define LITHE_ERR_ARG (-1)          /* invalid argument (shape, pointer, alignment)      */
#define LITHE_ERR_UNSUPPORTED (-2)  /* valid but not handled by this build (e.g. rank)   */
#define LITHE_ERR_CUDA (-3)         /* a CUDA runtime / driver call failed               */

/* bits of the device-side error word (int32) that kernels may OR in */
#define LITHE_DEVERR_SLOT 1         /* a sample referenced a slot >= n_slots             */
#define LITHE_DEVERR_INDEX 2        /* an int16/int32 bank held an index outside [0,512) */
#define LITHE_DEVERR_TIMEOUT 4      /* a pipeline wait ran past its time limit           */

#define LITHE_IDX_PACKED9 0         /* uint64 words, 7 x 9-bit, (block, level)-major     */
#define LITHE_IDX_I16 1             /* int16, level-major (slot, level, block)           */
#define LITHE_IDX_I32 2             /* int32, level-major (slot, level, block)           */

#define LITHE_DTYPE_BF16 0
#define LITHE_DTYPE_F32 1
#define LITHE_DTYPE_F16 2

#define LITHE_MAX_LEVELS 4

/* Where one side (A or B) of one module sits in a resident index bank.
 *   format LITHE_IDX_PACKED9: base = uint64 words of slot 0; slot s starts at
 *     base + s*slot_stride words; block j of this side has its level-l index at stream
 *     position offset + num_levels*j + l  (offset = num_levels * block offset of the side,
 *     i.e. 3*a_off / 3*b_off of PackedLayout, lithe/kernels/packed.py:100-117).
 *   format LITHE_IDX_I16 / LITHE_IDX_I32: element (s, l, j) is at
 *     base[s*slot_stride + offset + l*level_stride + j]. */
typedef struct lithe_index_view {
    const void* base;          /* device */
    int32_t format;            /* LITHE_IDX_* */
    int32_t num_levels;        /* L, 1..LITHE_MAX_LEVELS */
    int64_t slot_stride;       /* elements (words for PACKED9) between consecutive slots */
    int64_t offset;            /* see above */
    int64_t level_stride;      /* level-major formats only */
} lithe_index_view;

/* ABI version of this header; lithe_abi_version() returns the library's. */
#define LITHE_ABI_VERSION 1
LITHE_API int32_t lithe_abi_version(void);

/* Message for the last non-zero return on the calling thread ("" if none). */
LITHE_API const char* lithe_last_error(void);

/*
 * Fused index-resident per-sample LoRA forward for one linear (replaces the two Triton
 * launches of shared_codebook_lora_delta, lithe/kernels/shared.py:197-263, plus the
 * caller's "out + delta" pass, lithe/kernels/layers.py:131 and lithe/serve.py:97).
 *
 * For every sample b in [0, batch) with slot j = ids[b] (0 <= j < n_slots):
 *     A_j = decode(idx_a, j) reshaped (rank, d_in);  B_j = decode(idx_b, j) reshaped (d_out, rank)
 *     h   = bf16( w_b * scaling * (x[b] @ A_j^T) )             (fp32 accumulation)
 *     accumulate != 0:  out[b] = bf16( out[b] + h @ B_j^T )    (in place, fp32 add)
 *     accumulate == 0:  out[b] = bf16( h @ B_j^T )
 * where decode sums lut values over levels 0..L-1 in fp32 (lithe/quant.py:74-81) and
 * rounds to bf16 (the reference casts the decoded factors to the activation dtype,
 * lithe/serve.py:96).  w_b = weights[b] (weights may be NULL: w_b = 1).
 * ids[b] < 0: no adapter (out[b] untouched when accumulating, zero otherwise).
 * ids[b] >= n_slots: same as < 0 and LITHE_DEVERR_SLOT is OR-ed into *err_flag.
 *
 *   x    device bf16 (batch, m, d_in) contiguous;  out device bf16 (batch, m, d_out)
 *   ids  device int32 (batch);  weights device fp32 (batch) or NULL
 *   lut  HOST fp32 [2][num_levels][10]: side A levels then side B levels
 *   err_flag device int32 (may be NULL)
 * Requirements: rank in {1,2,4,8,16}; d_in % 64 == 0; d_out % 8 == 0; (d_out*rank) % 64 == 0;
 * x, out 16-byte aligned; idx_a and idx_b with the same num_levels.
 * m <= 8 (one decode step, per-sample modulation rows) runs a small-m kernel that splits the
 * output columns over CTAs; same formula and rounding steps, in every sgmv entry point.
 */
LITHE_API int32_t lithe_sgmv_index(const void* x, void* out, int32_t accumulate,
                         const lithe_index_view* idx_a, const lithe_index_view* idx_b,
                         int64_t n_slots, const int32_t* ids, const float* weights,
                         int32_t batch, int32_t m, int32_t d_in, int32_t d_out, int32_t rank,
                         const float* lut, float scaling, int32_t* err_flag, void* stream);

/*
 * lithe_sgmv_index with the element types given: x (and out when accumulating) in
 * x_dtype = LITHE_DTYPE_BF16 or LITHE_DTYPE_F16, the decoded factors, h and the MMAs in that
 * type (fp32 accumulation); out_dtype is x_dtype, or LITHE_DTYPE_F32 when accumulate == 0
 * (the delta alone, written in fp32 without a rounding to 16 bits).  Replaces the dtype
 * handling of shared_codebook_lora_delta (lithe/kernels/shared.py:210-218: pools cast to
 * x.dtype, the delta in out_dtype, default x.dtype).  Other combinations return
 * LITHE_ERR_UNSUPPORTED.  lithe_sgmv_index is this call with both dtypes LITHE_DTYPE_BF16.
 */
LITHE_API int32_t lithe_sgmv_index_typed(const void* x, void* out, int32_t accumulate,
                         const lithe_index_view* idx_a, const lithe_index_view* idx_b,
                         int64_t n_slots, const int32_t* ids, const float* weights,
                         int32_t batch, int32_t m, int32_t d_in, int32_t d_out, int32_t rank,
                         const float* lut, float scaling, int32_t x_dtype, int32_t out_dtype,
                         int32_t* err_flag, void* stream);

/* Bytes of device workspace lithe_sgmv_index_ws needs for a (batch, d_in, d_out) call:
 * batch * (d_in/64 + ceil(d_out/64)) * 512. */
LITHE_API int64_t lithe_sgmv_workspace_bytes(int32_t batch, int32_t d_in, int32_t d_out);

/*
 * lithe_sgmv_index in two launches on the same stream, with the same arguments, contract and
 * results (bit for bit).  A first kernel decodes every routed sample's A and B factors once
 * into `workspace` (512 bytes per 64-column chunk, 16 distinct values per block thanks to the
 * codebook's period-16 structure); the SGMV kernel then copies each chunk next to its
 * activation tile instead of re-decoding it for every 64-token tile.  Measured on B200 it is
 * slower than lithe_sgmv_index on every FLUX shape (the main loop pays a second bulk copy per
 * stage, more than the decode it saves); it is kept for callers that decode once and reuse the
 * workspace layout.  Replaces the same reference code as lithe_sgmv_index.
 *   workspace        device, 16-byte aligned, >= lithe_sgmv_workspace_bytes(batch, d_in, d_out);
 *                    contents on entry do not matter; calls sharing one workspace must be
 *                    ordered on one stream.
 */
LITHE_API int32_t lithe_sgmv_index_ws(const void* x, void* out, int32_t accumulate,
                         const lithe_index_view* idx_a, const lithe_index_view* idx_b,
                         int64_t n_slots, const int32_t* ids, const float* weights,
                         int32_t batch, int32_t m, int32_t d_in, int32_t d_out, int32_t rank,
                         const float* lut, float scaling, int32_t* err_flag,
                         void* workspace, int64_t workspace_bytes, void* stream);

/* Size of the built-in workspace of lithe_sgmv_index_noalloc (4 MiB per device). */
#define LITHE_NOALLOC_WS_BYTES (4LL << 20)

/*
 * lithe_sgmv_index_ws without the caller's workspace: an entry point that allocates no memory
 * of any kind.  It has no counterpart in the reference, which allocates its outputs and
 * scratch through PyTorch on every call.  It is meant for callers that cannot allocate device
 * memory on the request path: a C or C++ host that binds this library without PyTorch, whose
 * only allocator is cudaMalloc (which synchronises the device and can fail under memory
 * pressure in the middle of serving), or a serving loop that runs under a fixed memory budget.
 * The decoded factors go to a static device array of LITHE_NOALLOC_WS_BYTES that is part of the
 * library's image on each device; results equal lithe_sgmv_index's bit for bit.  Calls with
 * m <= 8 take the small-m form, which needs no workspace and leaves the array untouched.
 *   - Limit: lithe_sgmv_workspace_bytes(batch, d_in, d_out) must be <= LITHE_NOALLOC_WS_BYTES
 *     (e.g. batch 34 at d_in 3072, d_out 12288); a larger call returns LITHE_ERR_UNSUPPORTED
 *     and launches nothing.  Use lithe_sgmv_index or lithe_sgmv_index_ws for it.
 *   - Set-up: the first call in each CUDA context (in practice: on each device, whose primary
 *     context the runtime uses) looks up the array's device address with that context current
 *     (runtime calls, one of which initialises the context if needed); make that first call
 *     before any stream capture starts.  The address is cached per context handle.  After
 *     cudaDeviceReset() the device's next primary context may be given the old handle while the
 *     array sits at a new address, so do not call this entry point again in a process that has
 *     reset the device.
 *   - Nothing has to start at zero: every workspace byte the SGMV kernel reads is written by
 *     the same call's decode kernel.
 *   - Races: all calls on one device share the one array.  Two calls in flight at the same
 *     time on that device (different streams, or host threads without ordering) overwrite each
 *     other's factors; issue them on one stream or order them with events.
 */
LITHE_API int32_t lithe_sgmv_index_noalloc(const void* x, void* out, int32_t accumulate,
                         const lithe_index_view* idx_a, const lithe_index_view* idx_b,
                         int64_t n_slots, const int32_t* ids, const float* weights,
                         int32_t batch, int32_t m, int32_t d_in, int32_t d_out, int32_t rank,
                         const float* lut, float scaling, int32_t* err_flag, void* stream);

/*
 * Whole-adapter decode of a packed stream into dense 64-value blocks (replaces
 * _decode_packed_kernel / decode_packed, lithe/kernels/packed.py:151-177,205-222).
 *   words   device uint64, the packed (block, level)-major stream of one adapter
 *   n_blocks number of 64-value blocks (PackedLayout.total_blocks)
 *   sides   device int8 (n_blocks): 0 = A block, 1 = B block (NULL: all side A)
 *   lut     HOST fp32 [2][num_levels][10]
 *   out     device (n_blocks, 64) of out_dtype (LITHE_DTYPE_BF16 or LITHE_DTYPE_F32)
 * The fp32 output equals lithe.quant.rvq_decode_blocks bit for bit; the bf16 output is
 * that value rounded to nearest even.
 */
LITHE_API int32_t lithe_decode_packed(const uint64_t* words, int64_t n_blocks, int32_t num_levels,
                            const int8_t* sides, const float* lut, void* out,
                            int32_t out_dtype, void* stream);

/*
 * Batched decode of n_sel slots of a resident packed bank in one launch (the hot-swap /
 * decode-throughput path, serving/_common.py:241-244 run once per slot in the reference).
 *   bank      device uint64, slot s at bank + s*slot_stride words
 *   slot_ids  device int32 (n_sel): slots to decode (ids outside [0, n_slots) set
 *             LITHE_DEVERR_SLOT in *err_flag and leave their output rows untouched)
 *   out       device (n_sel, n_blocks, 64) of out_dtype
 */
LITHE_API int32_t lithe_decode_packed_batch(const uint64_t* bank, int64_t slot_stride, int64_t n_slots,
                                  const int32_t* slot_ids, int32_t n_sel, int64_t n_blocks,
                                  int32_t num_levels, const int8_t* sides, const float* lut,
                                  void* out, int32_t out_dtype, int32_t* err_flag, void* stream);

/*
 * Operands of lithe_lora_gemm's fused expand, for one linear (rank 16; same arguments and
 * routing as lithe_sgmv_index):
 *   h      device bf16 (batch * m, 16): h[b*m + i] = bf16( w_b * scaling * x[b, i] @ A_j^T ),
 *          the same values lithe_sgmv_index feeds its expand; zero rows for unrouted samples
 *   b_dec  device bf16 (batch, d_out, 16): B_j of every sample, decoded and rounded to bf16
 *          (zero for unrouted samples)
 * Two launches on `stream`: the B decode and the fused kernel in shrink-only form (x is read
 * once, no output tiles).  Either output may be NULL to skip its half (not both): split targets
 * of one fused Kohya module share A, so one h serves all of them.
 */
LITHE_API int32_t lithe_lora_prep(const void* x, const lithe_index_view* idx_a, const lithe_index_view* idx_b,
                        int64_t n_slots, const int32_t* ids, const float* weights, int32_t batch, int32_t m,
                        int32_t d_in, int32_t d_out, int32_t rank, const float* lut, float scaling, void* h,
                        void* b_dec, int32_t* err_flag, void* stream);

/* Bytes of device workspace lithe_lora_prep_ws needs for a (batch, m, d_in) call on the current
 * device: 8192 bytes per CTA of its shrink launch, min(SM count, batch * ceil(m/64) *
 * ceil(d_in/128)).  0 for an empty call; a negative LITHE_ERR_* code when the device cannot be
 * queried. */
LITHE_API int64_t lithe_lora_prep_workspace_bytes(int32_t batch, int32_t m, int32_t d_in);

/*
 * lithe_lora_prep with the shrink's work split evenly over the SMs: its CTAs take equal runs of
 * the (64-token tile, 128-column x stage) sequence instead of whole 64-token tiles, so a tile
 * may be shared by neighbouring CTAs.  Each stores its fp32 partial h of a shared tile in
 * `workspace`; the B-decode launch, which here follows the shrink on `stream`, adds the pieces
 * in CTA order, scales, rounds to bf16 and writes those tiles' h, so h does not depend on
 * timing.  h equals lithe_lora_prep's up to the fp32 summation order (one bf16 rounding step
 * at most); b_dec is identical.  Same arguments and outputs as lithe_lora_prep; the B-decode
 * kernel is launched even when b_dec is NULL if a tile is shared.  It pays where whole tiles
 * would load the SMs unevenly (at B=14 x 4096 tokens: 896 tiles over 148 SMs) and the x row
 * is long (d_in >= 12288); the Python host chooses it by that rule.  Replaces the same
 * reference code as lithe_lora_prep.
 *   workspace        device, 16-byte aligned, >= lithe_lora_prep_workspace_bytes(batch, m, d_in);
 *                    contents on entry do not matter; calls sharing one workspace must be
 *                    ordered on one stream.  Unused (may be NULL) when h is NULL.
 */
LITHE_API int32_t lithe_lora_prep_ws(const void* x, const lithe_index_view* idx_a, const lithe_index_view* idx_b,
                        int64_t n_slots, const int32_t* ids, const float* weights, int32_t batch, int32_t m,
                        int32_t d_in, int32_t d_out, int32_t rank, const float* lut, float scaling, void* h,
                        void* b_dec, int32_t* err_flag, void* workspace, int64_t workspace_bytes,
                        void* stream);

/* Bytes of device workspace lithe_lora_prep_multi needs: batch * (d_in/64) * n_targets * 512. */
LITHE_API int64_t lithe_lora_prep_multi_workspace_bytes(int32_t batch, int32_t d_in, int32_t n_targets);

/*
 * lithe_lora_prep for n_targets (1..4) rank-16 linears that read the same x (the q, k and v
 * projections of one attention block, each with its own adapter module): x is read once for
 * all of them.  Per target t, the same outputs and values as lithe_lora_prep with idx_a[t],
 * idx_b[t], d_out[t] and scaling[t]: h[t] (batch * m, 16) and b_dec[t] (batch, d_out[t], 16),
 * b_dec[t] may be NULL.  Two launches on `stream`: one decodes every routed sample's A chunks
 * of every target into `workspace` (plus the b_dec asked for); the shrink then streams each
 * x tile once and bulk-copies the targets' decoded chunks beside it.  Replaces the reference's
 * per-linear shrink (lithe/kernels/shared.py:36-95) called once per target on the same input.
 *   idx_a, idx_b, d_out, scaling, h, b_dec   HOST arrays of n_targets entries
 *   workspace        device, 16-byte aligned, >= lithe_lora_prep_multi_workspace_bytes(batch,
 *                    d_in, n_targets); contents on entry do not matter; calls sharing one
 *                    workspace must be ordered on one stream.
 */
LITHE_API int32_t lithe_lora_prep_multi(const void* x, int32_t n_targets, const lithe_index_view* idx_a,
                        const lithe_index_view* idx_b, const int32_t* d_out, int64_t n_slots, const int32_t* ids,
                        const float* weights, int32_t batch, int32_t m, int32_t d_in, int32_t rank,
                        const float* lut, const float* scaling, void* const* h, void* const* b_dec,
                        int32_t* err_flag, void* workspace, int64_t workspace_bytes, void* stream);

/*
 * Base linear with the per-sample LoRA expand inside the GEMM (tcgen05, TMEM accumulators, TMA):
 *   out[r, :] = x[r, :] . w^T + bias + h[r, :] . b_dec[r / rows_per_sample]^T
 * Replaces nn.Linear's GEMM + the delta's read-modify-write pass of the output
 * (lithe/kernels/layers.py:131, lithe/serve.py:96-97) for layers whose shapes it supports.
 *   x        device bf16 (rows, k), k-contiguous        w     device bf16 (n, k) (nn.Linear weight)
 *   bias     device bf16 (n) or NULL                      out   device bf16 (rows, n), written
 *   h        device bf16 (rows, rank): the scaled, bf16-rounded shrink (lithe_lora_prep), or NULL
 *            for the plain GEMM
 *   b_dec    device bf16 (rows / rows_per_sample, n, rank): every sample's decoded B factor
 * n must be a multiple of 256, k of 64; with h, rank 16 and rows_per_sample a multiple of 128
 * dividing rows (otherwise LITHE_ERR_UNSUPPORTED: use cuBLAS + lithe_sgmv_index).
 */
LITHE_API int32_t lithe_lora_gemm(const void* x, const void* w, const void* bias, void* out, int32_t rows, int32_t n,
                        int32_t k, const void* h, const void* b_dec, int32_t rows_per_sample, int32_t rank,
                        int32_t* err_flag, void* stream);

/* One (module, side) of a .lithe payload: its packed blocks [first_block, first_block + n_blocks)
 * come from raw[raw_offset + level * n_blocks + j], j = block - first_block. */
typedef struct {
    int64_t raw_offset;
    int64_t first_block;
    int64_t n_blocks;
} lithe_pack_segment;

/*
 * Pack a raw .lithe index payload into one bank slot on the device (replaces the host-side
 * load_lithe -> flat_indices -> pack_indices chain, lithe/fileio.py:119-152 and
 * lithe/kernels/packed.py:38-52,125-143, that the reference runs for every adapter it makes
 * resident).
 *   raw        device uint16 (n_raw): every module's A matrix in header order, then every
 *              module's B matrix, each (num_levels, n_blocks) row-major (the decompressed payload)
 *   segments   device, n_segments entries sorted by first_block, covering blocks
 *              [0, n_raw / num_levels) in packed (module A, module B, ...) order
 *   words      device uint64 (n_words = ceil(n_raw / 7)), e.g. a bank slot
 * Values above 511 and blocks the table does not cover set LITHE_DEVERR_INDEX in *err_flag
 * (the value is masked to 9 bits / written as 0).  No allocation, no host synchronisation.
 */
LITHE_API int32_t lithe_pack_raw(const uint16_t* raw, int64_t n_raw, const lithe_pack_segment* segments,
                       int32_t n_segments, int32_t num_levels, uint64_t* words, int64_t n_words,
                       int32_t* err_flag, void* stream);

/*
 * lithe_pack_raw for n_payloads payloads in one launch (a bulk load of payloads already on the
 * device): payload y at raw + y * raw_stride goes to bank slot slot_ids[y] (slot y when
 * slot_ids is NULL), i.e. bank + slot * slot_stride words.  Slots outside [0, n_slots) set
 * LITHE_DEVERR_SLOT and are skipped.  n_payloads <= 65535; raw_stride >= n_raw, a multiple of 8.
 */
LITHE_API int32_t lithe_pack_raw_batch(const uint16_t* raw, int64_t raw_stride, int32_t n_payloads, int64_t n_raw,
                             const lithe_pack_segment* segments, int32_t n_segments, int32_t num_levels,
                             uint64_t* bank, int64_t slot_stride, int64_t n_slots, const int32_t* slot_ids,
                             int64_t n_words, int32_t* err_flag, void* stream);

/*
 * Self-test of the bounded pipeline wait (no counterpart in the reference): one warp waits on
 * an mbarrier that nothing arrives at.  After the wait's time limit (4 s) it ORs
 * LITHE_DEVERR_TIMEOUT into *err_flag, writes 0 to *waited_ok (device int32, may be NULL) and
 * returns; the context stays usable.  This is the path every kernel's waits take when a
 * pipeline stalls, exercised without any fault.
 */
LITHE_API int32_t lithe_selftest_wait_timeout(int32_t* err_flag, int32_t* waited_ok, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* LITHE_B200_H */
