/*
 * mxwave_b200 -- C ABI of the B200 (sm_100a) MxWave hot path.
 *
 * Every entry point takes plain device pointers, sizes and a cudaStream_t
 * passed as `void*` (NULL = the legacy default stream), launches asynchronously
 * on that stream, allocates nothing, and returns an mxw_status code.  Argument
 * errors are detected on the host before any launch.  Kernels never trap; a
 * data-dependent failure (a NaN/inf weight) is reported through a caller-owned
 * device flag word that the caller reads when it next synchronises.
 *
 * Layouts follow the reference exactly:
 *   weight  [rows, cols] row-major, row stride `ld` elements (bf16/f16/f32)
 *   packed  [rows, cols/2] uint8, element 2j in the low nibble of byte j
 *   scales  [rows, cols/32] uint8, E8M0 biased exponent (exponent + 127)
 *   gamma   [cols] fp32;  hessian [cols/32, 32, 32] fp32
 * (compressed-tensors "mxfp4-pack-quantized", mxwave/core.py:147-149, 249-251)
 */
#ifndef MXWAVE_B200_H_
#define MXWAVE_B200_H_

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define MXW_API __attribute__((visibility("default")))
#else
#define MXW_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

/* Status codes. */
#define MXW_OK 0
#define MXW_EINVAL 1      /* bad argument (detected before launch)            */
#define MXW_ENONFINITE 2  /* reserved for callers mapping the flag word       */
#define MXW_ECUDA 3       /* a CUDA runtime call failed (see mxw_last_cuda_error) */
#define MXW_ETIMEOUT 4    /* a bounded device wait gave up                    */
#define MXW_EUNSUPPORTED 5

/* Element types of weight / activation inputs. */
#define MXW_BF16 0
#define MXW_F16 1
#define MXW_F32 2

/* Scale-selection methods (mxwave/core.py:22). */
#define MXW_METHOD_MSE 0
#define MXW_METHOD_RTN 1

/* Hessian damping modes (mxwave/core.py:23). */
#define MXW_DAMP_ABSOLUTE 0
#define MXW_DAMP_RELATIVE 1

/* Bits of the device flag word written by the kernels. */
#define MXW_FLAG_NONFINITE 1 /* the input held a NaN or infinity                 */
#define MXW_FLAG_TIMEOUT 2   /* a bounded on-device wait gave up; output invalid */
#define MXW_FLAG_RARE 4      /* quantize: a block took the exact rare-block pass  */

/* Human-readable name of a status code. */
MXW_API const char* mxw_status_string(int status);

/* The cudaError_t of the last MXW_ECUDA returned on this host thread. */
MXW_API int mxw_last_cuda_error(void);

/* Library version string. */
MXW_API const char* mxw_version(void);

/*
 * MXFP4 quantization of one row slice.
 * Replaces mxwave.core.quantize_mxfp4 (mxwave/core.py:114-251): percentile or
 * amax anchor, the explicit exponent candidate set floor-depth .. floor+1 plus
 * the no-clipping exponent, unweighted / gamma^2-weighted / block-Hessian
 * error, strict-< argmin (earliest candidate wins ties), E2M1 round-to-nearest
 * -even, nibble packing and E8M0 bytes.  method MXW_METHOD_RTN follows
 * _rtn_scale_exponent (core.py:91-104).  Output bytes are identical to the
 * reference's CPU fp32 implementation.
 *   gamma, hessian: device pointers or NULL (mutually exclusive; MSE only).
 *   flags: device uint32 word; MXW_FLAG_NONFINITE is OR-ed in when the slice
 *          holds a NaN or infinity (checkpoint.py:117), or NULL to skip.
 *          MXW_FLAG_RARE is OR-ed in when some block needs the exact second
 *          pass (non-finite values, magnitudes near FLT_MAX); with a flag word
 *          whose MXW_FLAG_RARE bit is clear after the main pass, the second
 *          pass returns at once instead of scanning the scale bytes.  The bit
 *          is sticky: a word shared by several calls only costs extra scans.
 */
MXW_API int mxw_quantize_mxfp4(const void* weight, int dtype, int64_t rows, int64_t cols, int64_t ld,
                       double scale_percentile, const float* gamma, const float* hessian,
                       int method, int mse_clip_depth, uint8_t* packed, uint8_t* scales,
                       uint32_t* flags, void* stream);

/*
 * Dequantize packed/scales to fp32 [rows, cols].
 * Replaces mxwave.core.dequant_mxfp4 (mxwave/core.py:254-278).
 */
MXW_API int mxw_dequant_mxfp4(const uint8_t* packed, const uint8_t* scales, int64_t rows, int64_t cols,
                      float* out, void* stream);

/*
 * Quantization-error sums for the SQNR family: one pass over an original
 * matrix [rows, cols] (row stride ld, dtype MXW_BF16/F16/F32) and its
 * reconstruction -- either a dense matrix (`reconstructed`, dtype rdtype, row
 * stride rld) or the packed MXFP4 bytes and E8M0 scales decoded on the fly
 * (packed/scales, cols % 32 == 0); exactly one of the two.  Writes
 *   sums[0] = sum o^2, sums[1] = sum (o - r)^2,
 *   sums[2], sums[3] = the same weighted by gamma^2 per input channel
 *   (gamma[cols]) or by the 32x32 block quadratic form (hessian[cols/32][32][32]),
 *   else 0.
 * fp64 accumulation with a fixed reduction order (bit-reproducible).
 * `workspace`: device memory of at least mxw_error_sums_workspace_size(rows,
 * cols) bytes, 16-byte aligned, whose first 16 bytes are zero before the first
 * call on it (each call leaves them zero again).  Calls sharing a workspace
 * must not overlap on the device.
 * Replaces the reductions of sqnr / channel_weighted_sqnr /
 * block_hessian_weighted_sqnr (mxwave/verify.py:24-86) and, with packed input,
 * the dequant_mxfp4 they follow in the engines (mxwave/engine.py:439-458).
 */
MXW_API size_t mxw_error_sums_workspace_size(int64_t rows, int64_t cols);
MXW_API int mxw_error_sums(const void* original, int dtype, int64_t rows, int64_t cols, int64_t ld,
                           const void* reconstructed, int rdtype, int64_t rld, const uint8_t* packed,
                           const uint8_t* scales, const float* gamma, const float* hessian, double* sums,
                           void* workspace, size_t workspace_bytes, void* stream);

/*
 * mxw_error_sums without a workspace, for callers that cannot allocate device
 * memory when they call: processes that reserve their whole device memory
 * budget at start-up and forbid later allocations (a serving process that has
 * carved up HBM, or a host application whose own pool owns every device
 * byte), and health checks that must still run when the device is out of
 * memory.  No counterpart in the reference.
 * Same arguments and results as mxw_error_sums minus the workspace.  Its
 * scratch is a fixed 65,552-byte device array in this library (a 16-byte
 * ticket plus fp64 partials for up to 2048 CTAs, i.e. 8 per SM on GPUs of up
 * to 256 SMs), held by every GPU that loads the library until the process
 * exits.  A launch that would need more scratch returns MXW_EUNSUPPORTED (use
 * mxw_error_sums with a workspace instead).  The call allocates nothing: it
 * clears the ticket with an asynchronous memset on `stream`, then launches.
 * Every call looks up the array's device address in the current context
 * (so it stays valid across cudaDeviceReset); the first call in a context may
 * load this library's kernels onto the device: make that first call before
 * any stream capture.  All calls share the one array, so calls that overlap
 * on the device (other streams, other host threads) race and must not be
 * issued concurrently.
 */
MXW_API int mxw_error_sums_noalloc(const void* original, int dtype, int64_t rows, int64_t cols, int64_t ld,
                                   const void* reconstructed, int rdtype, int64_t rld, const uint8_t* packed,
                                   const uint8_t* scales, const float* gamma, const float* hessian, double* sums,
                                   void* stream);

/*
 * Routing-weighted squared activations per expert: for every route r (row
 * route_rows[r] of x [rows, cols], row stride ld, squared router weight
 * route_w2[r]) adds fl(fl(x^2) * w2) into squares[e][cols] of its expert e,
 * and w2 into mass[e] (mass may be NULL).  Routes are grouped by expert:
 * those of expert e are [offsets[e], offsets[e+1]) of the n_routes entries,
 * in route order.  Sums are fp64 in route order, added once per expert and
 * column (deterministic).  Rows outside x and offsets outside [0, n_routes]
 * are ignored.
 * Replaces the index_add_ accumulations of RoutedLayerMoments.update_inputs
 * and update_down (mxwave/routed_calibration.py:104-141).
 */
MXW_API int mxw_accumulate_routed_squares(const void* x, int dtype, int64_t rows, int64_t cols, int64_t ld,
                                          const int64_t* route_rows, const float* route_w2, int64_t n_routes,
                                          const int64_t* offsets, int64_t experts, float* squares, float* mass,
                                          void* stream);

/*
 * Lossless repack of packed [rows, cols/2] MXFP4 codes and E8M0 scales
 * [rows, cols/32] (compressed-tensors layout; packed 16-byte aligned) into
 * ggml block_mxfp4 records: out[rows * cols/32 * 17] bytes, per block the
 * scale byte then 16 bytes holding element j (low nibble) and j + 16 (high).
 * Replaces repack_mxfp4_blocks (mxwave/gguf.py:134-150).
 */
MXW_API int mxw_repack_gguf_mxfp4(const uint8_t* packed, const uint8_t* scales, int64_t rows, int64_t cols,
                                  uint8_t* out, void* stream);

/*
 * Per-channel moments of activations x [tokens, cols] (row stride ld), added
 * into sum_abs[cols] (sum |x|) and sum_sq[cols] (sum x^2); either may be NULL.
 * Replaces the mean-abs / rms accumulation of ActivationCollector.update
 * (mxwave/calibration.py:227-232).
 */
MXW_API int mxw_accumulate_moments(const void* x, int dtype, int64_t tokens, int64_t cols, int64_t ld,
                           float* sum_abs, float* sum_sq, void* stream);

/*
 * Diagonal 32x32 blocks of X^T X added into gram_blocks [cols/32, 32, 32].
 * Replaces the block-hessian accumulation of ActivationCollector.update
 * (mxwave/calibration.py:233-236, einsum "nbi,nbj->bij").
 */
MXW_API int mxw_accumulate_block_gram(const void* x, int dtype, int64_t tokens, int64_t cols, int64_t ld,
                              float* gram_blocks, void* stream);

/*
 * One pass over x computing any subset of sum_abs / sum_sq (as
 * mxw_accumulate_moments) and gram_blocks (as mxw_accumulate_block_gram);
 * NULL outputs are skipped.  ActivationCollector.update with several
 * objectives (mxwave/calibration.py:226-236) reads its input once this way.
 * flags: device uint32 word for MXW_FLAG_TIMEOUT, or NULL.
 */
MXW_API int mxw_accumulate_activation_stats(const void* x, int dtype, int64_t tokens, int64_t cols,
                                    int64_t ld, float* sum_abs, float* sum_sq,
                                    float* gram_blocks, uint32_t* flags, void* stream);

/*
 * Full X^T X of bf16 activations x [tokens, cols] (row stride ld elements),
 * fp32 accumulation on the tcgen05 tensor cores, added into gram [cols, cols]
 * (row stride ldg).  The reference forms only the diagonal 32x32 blocks
 * (mxwave/calibration.py:233-236, core.py:55-56); the full product is the
 * calibration workload of the Hessian objective.  Requires cols % 128 == 0,
 * ld % 8 == 0, 16-byte aligned x and gram.  flags: MXW_FLAG_TIMEOUT or NULL.
 */
MXW_API int mxw_accumulate_xtx(const void* x, int64_t tokens, int64_t cols, int64_t ld, float* gram,
                               int64_t ldg, uint32_t* flags, void* stream);

/*
 * The same product in the kernel's packed form, for token-sharded callers
 * that all-reduce it: only the 128 x 256 tiles that reach the upper triangle,
 * each stored row-major and added into its slot of `packed`
 * (mxw_xtx_packed_floats(cols) floats, 16-byte aligned, zeroed by the caller
 * before the first slice).  At cols = 5120 that is 420 tiles, 55 MB against
 * the full Gram's 105 MB.  mxw_xtx_unpack then adds the packed tiles into a
 * full Gram (the entries with column >= row and their transposes), giving
 * the bits mxw_accumulate_xtx gives for the same slices.  Same requirements
 * otherwise.  No counterpart in the reference, which forms only the diagonal
 * blocks (mxwave/calibration.py:233-236).
 */
MXW_API size_t mxw_xtx_packed_floats(int64_t cols);
MXW_API int mxw_accumulate_xtx_packed(const void* x, int64_t tokens, int64_t cols, int64_t ld, float* packed,
                                      uint32_t* flags, void* stream);
MXW_API int mxw_xtx_unpack(const float* packed, int64_t cols, float* gram, int64_t ldg, void* stream);

/*
 * For a reduce-scatter of the packed tiles: the number of packed tiles at
 * `cols` (each 128 x 256 floats), and the unpack of tiles first_tile ..
 * first_tile + n_tiles - 1 read from `packed` (which holds just those tiles,
 * in order) into a full Gram; tiles past the last one are ignored, so a rank
 * may hold padding.  After a reduce-scatter each rank unpacks its own band of
 * tiles and owns those entries of the summed Gram.  No counterpart in the
 * reference, which forms only the diagonal blocks (mxwave/calibration.py:233-236).
 */
MXW_API int64_t mxw_xtx_packed_tiles(int64_t cols);
MXW_API int mxw_xtx_unpack_tiles(const float* packed, int64_t first_tile, int64_t n_tiles, int64_t cols,
                                 float* gram, int64_t ldg, void* stream);

/*
 * mean_abs = sum_abs / count, rms = sqrt(sum_sq / count) (either output may be
 * NULL).  Replaces ActivationCollector.finalize for the moment objectives
 * (mxwave/calibration.py:262-266).
 */
MXW_API int mxw_finalize_moments(const float* sum_abs, const float* sum_sq, int64_t cols, int64_t count,
                         float* mean_abs, float* rms, void* stream);

/*
 * Block Hessian = G / count with diagonal damping (absolute: + damp; relative:
 * + damp * mean(block diagonal)).  `full` = 0: G is gram_blocks
 * [cols/32,32,32]; `full` = 1: G is a full [cols, cols] Gram with row stride
 * ldg whose diagonal 32x32 blocks are taken.  out: [cols/32, 32, 32].
 * Replaces ActivationCollector.finalize for "block-hessian"
 * (mxwave/calibration.py:267-270) and _damp_block_hessian (core.py:61-69).
 */
MXW_API int mxw_finalize_block_hessian(const float* gram, int full, int64_t cols, int64_t ldg,
                               int64_t count, double damp, int mode, float* out, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* MXWAVE_B200_H_ */
