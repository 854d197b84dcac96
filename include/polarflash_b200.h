/*
 * polarflash_b200.h -- C ABI of the B200 (sm_100a) compressed-linear library.
 *
 * The library computes y = W x directly from packed low-bit weights
 * (INT4/INT3/INT2 codes, E8 root residual-VQ indices, recursive polar
 * blocks), with the inverse block randomized Walsh-Hadamard transform of the
 * weight folded in as a forward transform of x.  Every pointer argument
 * named "device" must point into memory of the current CUDA device; every
 * launch goes to the caller's stream and returns without synchronising.
 * No entry point allocates device memory: scratch space is the caller's
 * `workspace` buffer (size from pf_qlinear_workspace_size).
 *
 * Errors: every entry point returns a pf_status.  Argument errors are found on
 * the host before anything is launched; PF_ERR_CUDA reports a launch failure
 * (cudaGetLastError) and pf_last_cuda_error() returns the CUDA error code.
 */
#ifndef POLARFLASH_B200_H
#define POLARFLASH_B200_H

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define PF_API __attribute__((visibility("default")))
#else
#define PF_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

/* Status codes (the Python layer maps them to ValueError / RuntimeError as
 * the reference does, polarflash_quant/unified_quantizer.py:100-101,
 * polarflash_rt/cuda/native_kernels.py:396-410). */
typedef enum pf_status {
  PF_OK = 0,
  PF_ERR_INVALID_ARGUMENT = 1, /* null pointer, unknown enum value          */
  PF_ERR_SHAPE = 2,            /* M, K or N outside what the format allows  */
  PF_ERR_ALIGNMENT = 3,        /* a device pointer is not aligned enough    */
  PF_ERR_UNSUPPORTED = 4,      /* format/parameter combination not built    */
  PF_ERR_WORKSPACE = 5,        /* workspace missing or too small            */
  PF_ERR_CUDA = 6,             /* CUDA launch / runtime failure             */
  PF_ERR_TIMEOUT = 7           /* a bounded device wait gave up             */
} pf_status;

/* Packed weight formats.  Codes of the reference formats are bit-identical
 * to the reference packers (polarflash_quant/bitpacking.py); the *_G128 and
 * E8 formats are extensions defined in the same conventions.
 *
 *  PF_FMT_INT4_G128  codes: u32 words, 8 codes per word (code i at bits 4i),
 *                    16 words per (row, 128-column group); scales, mins:
 *                    fp16 [M][K/128]; w = q*s + m (the asymmetric convention of
 *                    polarflash_rt/kv_cache/compressed_kv.py:115-146).
 *  PF_FMT_INT3_G128  10 codes per word (code i at bits 3i, bits 30-31 zero),
 *                    13 words per (row, group); scales/mins as INT4_G128.
 *  PF_FMT_INT2_G128  16 codes per word (code i at bits 2i), 8 words per group.
 *  PF_FMT_INT4       reference pack_int4 stream (bitpacking.py:16-31), rows of
 *                    K/2 bytes; w = (code - 8) * scale.
 *  PF_FMT_INT3       reference pack_int3 stream (bitpacking.py:88-123), rows of
 *                    3K/8 bytes; w = (code - 4) * scale.
 *  PF_FMT_INT2       reference pack_int2 stream (bitpacking.py:49-65), rows of
 *                    K/4 bytes; w = (code - 2) * scale.
 *                    For the three reference INT formats `scale` is
 *                    tensor_scale (UnifiedQuantizer, unified_quantizer.py:154-178)
 *                    or, when `scales` is non-NULL, fp32 [M] per-row scales
 *                    (NativeLowBitCUDAEngine, native_kernels.py:415-576).
 *  PF_FMT_E8_RVQ2_G128  idx: u8 [M][K/8][2] (stage-interleaved root indices in
 *                    generate_e8_roots order, e8_lattice.py:21-50); scales: fp16
 *                    [M][K/128][2]; w8 = s1*r[i1] + s2*r[i2].
 *  PF_FMT_POLAR_RECURSIVE  encode_packed stream (polar_quant.py:381-487):
 *                    MSB-first blocks of params[1..d] bits, rows of K/d blocks;
 *                    params[0] = d (block size), params[1..d] = allocation;
 *                    tensor_scale = r_scale.  scales: NULL (uniform angle
 *                    grid), or for a weight encoded with learned angle
 *                    codebooks (fit_codebooks, polar_quant.py:274-300) fp32
 *                    [d-1][64]: entry 64 j + c is the angle of code c in angle
 *                    column j (level 0 columns first), i.e. the codebook of
 *                    j's level at min(c, codebook length - 1)
 *                    (decode_packed, polar_quant.py:552-554).
 *  PF_FMT_POLAR2D    2-D polar pairs (polar_quant.py:18-73): MSB-first
 *                    (r << theta_bits | theta); params[0] = r_bits,
 *                    params[1] = theta_bits; tensor_scale = r_scale.
 */
typedef enum pf_format {
  PF_FMT_INT4_G128 = 1,
  PF_FMT_INT3_G128 = 2,
  PF_FMT_INT2_G128 = 3,
  PF_FMT_INT4 = 4,
  PF_FMT_INT3 = 5,
  PF_FMT_INT2 = 6,
  PF_FMT_E8_RVQ2_G128 = 7,
  PF_FMT_POLAR_RECURSIVE = 8,
  PF_FMT_POLAR2D = 9
} pf_format;

typedef enum pf_dtype { PF_DTYPE_F32 = 0, PF_DTYPE_F16 = 1, PF_DTYPE_BF16 = 2 } pf_dtype;

/* A packed weight resident on the device.  Replaces the (raw_bytes,
 * quant_meta) pair that PolarLinearLayer keeps (polarflash_rt/cpu/engine.py:36-56). */
typedef struct pf_qweight {
  int32_t format;            /* pf_format                                      */
  int32_t M;                 /* out_features (rows of W)                       */
  int32_t K;                 /* in_features (columns of W)                     */
  int32_t had_block;         /* RWHT block the weight was rotated with; 0 = none
                                (hadamard_block_size after _init_dims,
                                polarflash_quant/transforms/hadamard.py:93-99) */
  const void* codes;         /* device: packed payload                         */
  const void* scales;        /* device: per format (see above), may be NULL    */
  const void* mins;          /* device: fp16 group mins for *_G128, else NULL  */
  const int8_t* had_signs;   /* device: K per-column signs (+1/-1), or NULL    */
  double tensor_scale;       /* per-tensor scale / polar r_scale               */
  int32_t params[20];        /* format parameters (polar block size, alloc)    */
} pf_qweight;

/* Library identity. */
PF_API const char* pf_version(void);
PF_API const char* pf_status_string(int status);
PF_API int pf_last_cuda_error(void);
/* Kernel launches this library has issued in this process, over all devices
 * and streams.  A launch recorded into a CUDA graph counts once, at capture;
 * graph replays add nothing. */
PF_API unsigned long long pf_kernel_launches(void);

/* Checks a descriptor (shapes, pointers, alignment) without launching. */
PF_API int pf_qweight_check(const pf_qweight* w);

/* Bytes of device workspace pf_qlinear needs for N input rows.  The
 * workspace holds a block of split-K arrival counters at its start, split-K
 * partial sums and, for the formats that need one, the prepared activations.  Zero-fill a workspace once
 * after allocating it; every call leaves the counters zero again.  Calls
 * that share one workspace must be ordered (same stream). */
PF_API int pf_qlinear_workspace_size(const pf_qweight* w, int N, size_t* bytes);

/* y[N][M] (fp32) = x[N][K] * W^T (+ bias[M]).  Replaces PolarLinearLayer.forward
 * (polarflash_rt/cpu/engine.py:90-96) and, through it, PFlashCUDAEngine.forward_layer
 * (polarflash_rt/cuda/engine.py:129-145): the dequantize -> inverse RWHT ->
 * torch.matmul chain becomes one fused launch sequence on `stream`.
 * x: device, dtype pf_dtype, row-major [N][K]; bias: device fp32 [M] or NULL;
 * y: device fp32 [N][M]; workspace: device, 256-byte aligned. */
PF_API int pf_qlinear(const pf_qweight* w, const void* x, int x_dtype, int N, const float* bias,
               float* y, void* workspace, size_t workspace_bytes, void* stream);

/* `count` linears in one call: y_i[N][M_i] = x_i[N][K_i] * W_i^T (+ bias_i),
 * i < count (no counterpart in the reference, whose layers run one at a
 * time; used where a model feeds one input to several weights: q/k/v,
 * gate/up).  When every weight takes the streaming GEMV (INT formats with
 * K % 512 == 0, one format and scale mode, rotation block <= 512, x 16-byte
 * aligned for fp32 or 8-byte for fp16/bf16), each 16-token pass of up to four
 * weights is ONE kernel launch; otherwise the weights run one after another
 * as pf_qlinear.  ws, xs, biases (may be NULL, or hold NULLs) and ys are host
 * arrays of `count` entries; the pointers they hold are device pointers. */
PF_API int pf_qlinear_group_workspace_size(int count, const pf_qweight* const* ws, int N, size_t* bytes);
PF_API int pf_qlinear_group(int count, const pf_qweight* const* ws, const void* const* xs, int x_dtype, int N,
                            const float* const* biases, float* const* ys, void* workspace,
                            size_t workspace_bytes, void* stream);

/* pf_qlinear for callers that cannot allocate device memory (no counterpart
 * in the reference, which has no GPU linear of its own to mirror here).
 * Same inputs, outputs and semantics as pf_qlinear, but the scratch space
 * comes from a fixed 8 MiB array inside the library's device image, reserved
 * on every GPU that loads the library until the process exits; no device
 * memory is allocated.  A request is refused with PF_ERR_WORKSPACE when even
 * the least workspace pf_qlinear accepts for it (smaller than
 * pf_qlinear_workspace_size for batches above 16 tokens) exceeds 8 MiB;
 * batches above 16 tokens then run the tensor-core GEMM without its stream-K
 * partial tiles.  The first call on a device looks up the array's address,
 * zeroes its counters and waits for the device, so make it before any stream
 * capture.  All calls on a device share the array: calls that overlap on the
 * GPU (unordered streams) race on it. */
PF_API int pf_qlinear_noalloc(const pf_qweight* w, const void* x, int x_dtype, int N, const float* bias,
                              float* y, void* stream);

/* Device status after the work queued on `stream` (the call synchronises
 * the stream).  Every device wait of this library's kernels is bounded: a
 * wait that runs out records PF_ERR_TIMEOUT in the workspace's status word
 * and the kernel finishes early with incomplete outputs, after its launch
 * already returned PF_OK.  *status receives PF_OK or the recorded PF_ERR_*;
 * *busy_counters (may be NULL) the number of split-K arrival counters not
 * back at zero (0 after every completed call); `reset` non-zero zeroes the
 * status word and the counters again so the workspace can be reused.  The
 * reference surfaces driver failures as RuntimeError
 * (polarflash_rt/cuda/native_kernels.py:396-410); the Python layer raises it
 * from this status.  pf_qlinear_noalloc_status does the same for the
 * library-held scratch array of pf_qlinear_noalloc on the current device. */
PF_API int pf_workspace_status(void* workspace, int reset, int* status, int* busy_counters, void* stream);
PF_API int pf_qlinear_noalloc_status(int reset, int* status, int* busy_counters, void* stream);
/* Runs the library's bounded device wait (the loop every streaming kernel
 * uses) on a barrier that no thread completes, with a limit of `wait_ns`
 * (0 < wait_ns <= 2e9): the wait runs out and records PF_ERR_TIMEOUT in the
 * workspace's status word, as a kernel that timed out does.  A diagnostic of
 * the timeout path for tests and deployment checks; no counterpart in the
 * reference. */
PF_API int pf_wait_selftest(void* workspace, unsigned long long wait_ns, void* stream);

/* ---- Column-parallel linears with the all-gather fused into the GEMV.
 *
 * Rank r of `world` holds rows [r M / world, (r + 1) M / world) of each
 * weight.  Instead of an all-gather after the GEMV, every rank's kernel
 * stores its output rows straight into every rank's peer buffer over NVLink
 * (plain peer stores, no multicast), then raises its flag in every buffer
 * and waits (bounded) for every rank's flag: when the call's kernels
 * complete on a rank, all ranks' rows are in its buffer.  pf_peers_wait
 * repeats that wait in a small kernel, for consumers on another stream.  The reference computes each
 * linear on one device (polarflash_rt/cuda/engine.py:129-145); this sharding
 * is the column-parallel form of that contract.
 *
 * A peer buffer is device memory of the same size on every rank (the caller
 * allocates it, zero-filled); its first 256 bytes are the header the calls
 * use (an epoch and one flag per rank), outputs live at byte offsets >= 256
 * that are the same on every rank.  pf_peer_export / pf_peer_open exchange
 * the buffers between the ranks' processes (CUDA IPC; the handle bytes are
 * passed through the caller's own channel, e.g. torch.distributed). */
typedef struct pf_peers {
  int32_t world;              /* ranks, 1..8                                   */
  int32_t rank;               /* this process's rank                           */
  void* bases[8];             /* device: each rank's peer buffer, mapped here  */
  size_t bytes;               /* size of every peer buffer                     */
} pf_peers;
/* 64-byte IPC handle of the allocation that holds `ptr`, and ptr's offset in it. */
PF_API int pf_peer_export(const void* ptr, unsigned char handle[64], size_t* offset);
/* Maps a peer's exported buffer into this process: *ptr = its base + offset.
 * *mapping receives the mapping to pass to pf_peer_close. */
PF_API int pf_peer_open(const unsigned char handle[64], size_t offset, void** ptr, void** mapping);
PF_API int pf_peer_close(void* mapping);
/* pf_qlinear_group on this rank's row shards ws[i] (M_i = m_full_i / world
 * rows each, a multiple of 128), with y of linear i written as
 * [N][m_full_i] fp32 at byte offset y_offsets[i] (16-byte aligned, >= 256)
 * of every rank's peer buffer, this rank's rows from row rank * M_i.  Takes
 * the streaming GEMV (group-128 INT formats, K % 512 == 0, N <= 16, x 16-byte
 * aligned); else PF_ERR_UNSUPPORTED.  Every rank makes the same sequence of
 * calls.  The workspace is pf_qlinear_group_workspace_size's. */
PF_API int pf_qlinear_group_gather(int count, const pf_qweight* const* ws, const void* const* xs, int x_dtype,
                                   int N, const float* const* biases, const size_t* y_offsets,
                                   const int* m_full, const pf_peers* peers, void* workspace,
                                   size_t workspace_bytes, void* stream);
/* All-gather of row shards that are already computed, over the same peer
 * buffers (replaces an ncclAllGather after a column-parallel linear whose
 * shard came from elsewhere; polarflash_rt/cuda/engine.py:129-145 computes
 * the whole y on one device).  This rank's `bytes` at `src` (device,
 * 16-byte aligned, a multiple of 16) land at byte dst_offset + rank * bytes
 * of every rank's buffer (rank-major, as ncclAllGather orders them;
 * dst_offset >= 256 and 16-byte aligned, world * bytes must fit).  One
 * kernel: plain peer stores, then the launch's last block raises this rank's
 * flag in every buffer and waits (bounded) for every rank's flag, so when the
 * kernel completes the gathered rows are in the local buffer.  Every rank
 * makes the same sequence of gathering calls. */
PF_API int pf_allgather_rows(const pf_peers* peers, const void* src, size_t bytes, size_t dst_offset,
                             void* workspace, void* stream);
/* Makes `stream` wait (one small kernel, each wait bounded to 2 s) until
 * every rank's rows of this rank's latest pf_qlinear_group_gather call are
 * in its peer buffer (the call's own kernel already waits for them; this is
 * for consumers ordered after it on another stream).  A wait that gives up
 * records PF_ERR_TIMEOUT in the workspace status word (pf_workspace_status). */
PF_API int pf_peers_wait(const pf_peers* peers, void* workspace, void* stream);

/* W_hat[M][K] (fp32) = decoded weight, followed by the inverse block RWHT
 * when `inverse_rwht` is non-zero and the weight is rotated.  Replaces
 * UnifiedQuantizer.dequantize (polarflash_quant/unified_quantizer.py:242-324). */
PF_API int pf_dequant(const pf_qweight* w, float* W_out, int inverse_rwht, void* stream);

/* Unpacked codes u8 [M][K] (bit-exact with the reference unpackers,
 * bitpacking.py:34-156) for the INT formats; E8: indices u8 [M][K/8][2]. */
PF_API int pf_unpack_codes(const pf_qweight* w, uint8_t* codes_out, void* stream);

/* Block randomized Walsh-Hadamard on rows of a [rows][K] fp32 matrix
 * (BlockHadamardTransform.forward / .inverse, hadamard.py:119-169).
 * signs: device, K per-column +-1 as int8; block: effective block size. */
PF_API int pf_rwht(const float* in, float* out, int rows, int K, int block, const int8_t* signs,
            int inverse, void* stream);

/* NativeLowBitCUDAEngine mirrors (polarflash_rt/cuda/native_kernels.py:415-576):
 * packed uint8 [M][K/2] (int4, nibble - 8) or [M][K/4] (int2, code - 2),
 * per-row fp32 scales [M], fp32 x / y, no rotation. */
PF_API int pf_native_gemv_int4(const float* x, const uint8_t* packed, const float* scales, int M,
                        int K, float* y, void* workspace, size_t workspace_bytes, void* stream);
PF_API int pf_native_gemv_int2(const float* x, const uint8_t* packed, const float* scales, int M,
                        int K, float* y, void* workspace, size_t workspace_bytes, void* stream);
PF_API int pf_native_gemm_int4(const float* X, const uint8_t* packed, const float* scales, int N,
                        int M, int K, float* Y, void* workspace, size_t workspace_bytes,
                        void* stream);

/* Decode-step helpers around the packed linears (batch 1, fp32 device
 * buffers; `pos` is a device int64 holding the new token's position, so a
 * whole step can be captured once as a CUDA graph).
 *
 * pf_add_rmsnorm: for each of `rows` rows of h [rows][H]: h += delta (if
 * delta is non-null, in place), out = h / sqrt(mean(h^2) + eps) * w.
 * Replaces the residual add of PFlashTransformerLayer.forward and
 * RMSNorm.forward (polarflash_core/model_integration.py:183-192, 34-37). */
PF_API int pf_add_rmsnorm(float* h, const float* delta, const float* w, float* out, int rows, int H, float eps,
                          void* stream);
/* pf_rope_kv: q [n_heads][head_dim] rotated in place, k [n_kv_heads][head_dim]
 * rotated into k_cache[*pos] and v copied into v_cache[*pos] (caches
 * [max_seq][n_kv_heads][head_dim]); angle = *pos * inv_freq[i] for the pair
 * (i, i + head_dim/2).  Replaces apply_rotary_pos_emb and the cache update of
 * PFlashAttentionBlock.forward (model_integration.py:40-60, 109-122). */
PF_API int pf_rope_kv(float* q, const float* k, const float* v, float* k_cache, float* v_cache,
                      const long long* pos, const float* inv_freq, int n_heads, int n_kv_heads, int head_dim,
                      int max_seq, void* stream);
/* pf_decode_attention: out [n_heads][head_dim] = softmax(q k^T * scale) v over
 * positions 0..*pos of the caches, query head h reading KV head
 * h / (n_heads / n_kv_heads); head_dim a multiple of 4 and <= 128, at most
 * 8 query heads per KV head, max_seq <= 32768; the caches 16-byte aligned
 * (rows are read as float4).  The positions are split into chunks of 64 whose
 * partial results go to `workspace` (device, at least
 * pf_decode_attention_workspace_size bytes) and are merged by a second
 * launch.  Replaces the GQA attention of PFlashAttentionBlock.forward
 * (model_integration.py:126-145) for one new token. */
PF_API size_t pf_decode_attention_workspace_size(int n_heads, int head_dim, int max_seq);
PF_API int pf_decode_attention(const float* q, const float* k_cache, const float* v_cache, const long long* pos,
                               float* out, int n_heads, int n_kv_heads, int head_dim, int max_seq, float scale,
                               void* workspace, size_t workspace_bytes, void* stream);
/* pf_silu_mul: out = silu(g) * u elementwise.  Replaces the gate of
 * PFlashMLPBlock.forward (model_integration.py:160-163). */
PF_API int pf_silu_mul(const float* g, const float* u, float* out, long long n, void* stream);

/* Compressed KV cache: rows of `dim` values (one token of one KV head)
 * stored as codes plus a per-row fp32 scale (and zero), as CompressedKVCache
 * quantizes them (polarflash_rt/kv_cache/compressed_kv.py):
 *   PF_KV_INT8 (:68-77):  s = max(max|x| / 127, 1e-8), int8 c = clamp(round(x / s), -128, 127),
 *                         x' = c s; dim bytes per row.
 *   PF_KV_2BIT (:79-112): s = max(max|x| / 1.75, 1e-8), c = clamp(floor(x / s + 2), 0, 3),
 *                         x' = (c - 1.5) s; (dim + 3) / 4 bytes per row.
 *   PF_KV_2BIT_ASYM (:114-150): z = min x, s = max((max x - z) / 3, 1e-8),
 *                         c = clamp(round((x - z) / s), 0, 3), x' = c s + z.
 * round is to nearest even; 2-bit codes are packed four per byte, first value
 * in the top bits (c0 << 6 | c1 << 4 | c2 << 2 | c3), a ragged last byte
 * padded with zero codes.  Codes, scales and x' are bit-identical to the
 * reference's fp32 arithmetic for finite inputs.  PF_KV_FP32 names the plain
 * fp32 cache of pf_rope_kv / pf_decode_attention. */
typedef enum pf_kv_mode { PF_KV_FP32 = 0, PF_KV_INT8 = 1, PF_KV_2BIT = 2, PF_KV_2BIT_ASYM = 3 } pf_kv_mode;
/* Bytes of one row of codes (4 * dim for PF_KV_FP32); 0 for a bad mode or dim. */
PF_API size_t pf_kv_row_bytes(int mode, int dim);
/* pf_kv_quantize: x [rows][dim] fp32 -> codes [rows][pf_kv_row_bytes],
 * scales [rows], zeros [rows] (PF_KV_2BIT_ASYM only; may be null otherwise).
 * The quantize half of CompressedKVCache.update (compressed_kv.py:152-259). */
PF_API int pf_kv_quantize(const float* x, long long rows, int dim, int mode, void* codes, float* scales,
                          float* zeros, void* stream);
/* pf_kv_dequantize: out [rows][dim] fp32 = x' of each row.  The dequantize
 * half of CompressedKVCache.update (_dequantize_*, compressed_kv.py:75-77,
 * 101-112, 139-150). */
PF_API int pf_kv_dequantize(const void* codes, const float* scales, const float* zeros, long long rows, int dim,
                            int mode, float* out, void* stream);
/* pf_rope_kv_compressed: as pf_rope_kv, with the rotated k and v quantized
 * (mode PF_KV_INT8 / PF_KV_2BIT / PF_KV_2BIT_ASYM) into row (*pos, head) of
 * compressed caches: codes [max_seq][n_kv_heads][pf_kv_row_bytes(mode,
 * head_dim)], scales and zeros [max_seq][n_kv_heads].  head_dim <= 2048. */
PF_API int pf_rope_kv_compressed(float* q, const float* k, const float* v, void* k_codes, float* k_scales,
                                 float* k_zeros, void* v_codes, float* v_scales, float* v_zeros,
                                 const long long* pos, const float* inv_freq, int n_heads, int n_kv_heads,
                                 int head_dim, int max_seq, int mode, void* stream);
/* pf_decode_attention_compressed: pf_decode_attention over compressed caches
 * laid out as pf_rope_kv_compressed writes them, each K and V value
 * dequantized inside the attention kernel (the reference dequantizes the
 * whole cache, compressed_kv.py:173-226, and attends over the result).
 * Same shape limits as pf_decode_attention; int8 codes 4-byte aligned. */
PF_API int pf_decode_attention_compressed(const float* q, const void* k_codes, const float* k_scales,
                                          const float* k_zeros, const void* v_codes, const float* v_scales,
                                          const float* v_zeros, const long long* pos, float* out, int n_heads,
                                          int n_kv_heads, int head_dim, int max_seq, int mode, float scale,
                                          void* workspace, size_t workspace_bytes, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* POLARFLASH_B200_H */
