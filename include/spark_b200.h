/*
 * spark_b200.h -- C ABI of the SPARK online-dequant linear path for B200
 * (sm_100a).  Plain pointers and sizes only; every buffer is owned by the
 * caller and every call is ordered on the caller's CUDA stream (`stream` is a
 * cudaStream_t passed as void*, NULL = legacy default stream).
 *
 * Return value: SPARK_OK (0), a negative SPARK_ERR_* for an invalid call
 * (nothing was launched), or a positive cudaError_t from the launch.  The
 * message of the last error on the calling thread is spark_last_error().
 *
 * Packed layouts are exactly the reference's on-disk formats (DJAzzs/SPARK):
 *   SPFP2 paired  01_core/block_fp2_emu.py:231-267  5 B per 16 weights
 *   SPFP2 v1      01_core/block_fp2_emu.py:86-167   3 B per 8 weights
 *   FP3 3-bit     01_core/fp3_emu.py:107-139        3 B per 8 codes + e4m3 scale / 16
 *   FP3 nibble    01_core/fp3_emu.py:50-73          1 B per 2 codes + e4m3 scale / 16
 *   NVFP4         01_core/nvfp4_emu.py:81-107       1 B per 2 codes + e4m3 scale / 16
 *   2:4 SPFP2     01_core/two_four.py:112-155       7 B per 32 weights
 */
#ifndef SPARK_B200_H
#define SPARK_B200_H

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define SPARK_API __attribute__((visibility("default")))
#else
#define SPARK_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

#define SPARK_OK 0
#define SPARK_ERR_INVALID (-1)     /* bad size, pointer or enum */
#define SPARK_ERR_ALIGNMENT (-2)   /* pointer or stride not aligned as required */
#define SPARK_ERR_UNSUPPORTED (-3) /* valid request this build does not implement */
#define SPARK_ERR_WORKSPACE (-4)   /* workspace missing or too small */
#define SPARK_ERR_DEVICE (-5)      /* a kernel reported an error through its workspace flag */

/* element types of float tensors */
#define SPARK_DTYPE_F32 0
#define SPARK_DTYPE_BF16 1
#define SPARK_DTYPE_F16 2

/* packed weight formats accepted by the linear entry points */
#define SPARK_FMT_SPFP2 0    /* paired, 5 B / 16 weights (the container's *_packed) */
#define SPARK_FMT_SPFP2_V1 1 /* 3 B / 8 weights (_detect_format "v1") */
#define SPARK_FMT_FP3 2      /* 3-bit codes + e4m3 scales (the container's *_fp3_codes/_fp3_scales) */
#define SPARK_FMT_NVFP4 3    /* e2m1 nibbles + e4m3 scales (*_nvfp4_codes/_nvfp4_scales) */
#define SPARK_FMT_TWOFOUR 4  /* 2:4-sparse SPFP2, 7 B / 32 weights ("v3-24") */
/* OR'ed into a format: the weight buffer holds the fragment-major ("tiled")
 * copy made by spark_tile_weights (scales embedded) instead of the reference layout */
#define SPARK_LAYOUT_TILED 0x100
/* spark_linear flag: run the tcgen05 kernel (SPFP2 reference layout, bf16 x,
 * ic a multiple of 256, 16-byte aligned weights and x, ldx a multiple of 8);
 * SPARK_ERR_UNSUPPORTED when the call does not meet those conditions. */
#define SPARK_PATH_TCGEN05 0x200
/* Fused MLP activation: the weight's rows come in 16-row groups of 8 gate rows
 * then the matching 8 up rows (V3GateUpSiLU builds this order); y gets
 * SiLU(gate) * up, oc / 2 columns wide.  Decode GEMV paths only. */
#define SPARK_EPILOGUE_SILU 0x400

SPARK_API const char* spark_last_error(void);
SPARK_API int spark_version(void);

/* ---------------------------------------------------------------- SPFP2 */
/* pack_blockwise_paired(w) -- 01_core/block_fp2_emu.py:231.
 * w: n floats (dtype), n % 8 == 0, blocks of 8 over the flattened tensor.
 * packed: ceil(n/16)*5 bytes; expv: n/8 bytes (may be NULL). */
SPARK_API int spark_spfp2_pack(const void* w, int w_dtype, int64_t n, uint8_t* packed, uint8_t* expv, void* stream);
/* pack_blockwise_search(w, window=2) -- 01_core/block_fp2_emu.py:86.  packed: n/8*3 bytes. */
SPARK_API int spark_spfp2_pack_v1(const void* w, int w_dtype, int64_t n, uint8_t* packed, uint8_t* expv, void* stream);
/* unpack_blockwise_paired(packed, n_elements) -- 01_core/block_fp2_emu.py:270. */
SPARK_API int spark_spfp2_unpack(const uint8_t* packed, int64_t n_elements, void* out, int out_dtype, void* stream);
/* The legacy single-exponent layout (5 B per 16 weights: 32-bit code word + exponent in
 * the low nibble of byte 4) -- replaces spark_decode_launch_f32/f16
 * (01_core/block_fp2_kernel.cu:67-87, kernels :3-62) behind the decode_fp32/decode_fp16
 * torch ops (01_core/build_spark_fp2.py:28-54).  out: 16 * n_blocks values. */
SPARK_API int spark_spfp2_legacy_decode(const uint8_t* packed, int64_t n_blocks, void* out, int out_dtype,
                                        void* stream);
/* unpack_blockwise(packed) (3-byte) -- 01_core/block_fp2_emu.py:204. */
SPARK_API int spark_spfp2_unpack_v1(const uint8_t* packed, int64_t n_blocks, void* out, int out_dtype, void* stream);
/* channel_fake_quantize(w) forward -- 01_core/block_fp2_emu.py:365 (STE backward is the
 * identity, :359-362). */
SPARK_API int spark_spfp2_fake_quant(const void* w, int w_dtype, int64_t n, void* out, int out_dtype, void* stream);

/* ---------------------------------------------------------------- FP3 E1M1 */
/* fp3_pack_3bit(w) -- 01_core/fp3_emu.py:107.  w: [oc, ic]; codes: ceil(oc*ceil(ic/16)*16/8)*3 B;
 * scales: oc*ceil(ic/16) e4m3 bytes. */
SPARK_API int spark_fp3_pack(const void* w, int w_dtype, int64_t oc, int64_t ic, uint8_t* codes, uint8_t* scales,
                   void* stream);
/* fp3_pack(w) (nibble codes) -- 01_core/fp3_emu.py:50.  codes: ceil(n/2) B. */
SPARK_API int spark_fp3_pack_nibble(const void* w, int w_dtype, int64_t oc, int64_t ic, uint8_t* codes, uint8_t* scales,
                          void* stream);
/* fp3_unpack_3bit -- 01_core/fp3_emu.py:142. */
SPARK_API int spark_fp3_unpack(const uint8_t* codes, const uint8_t* scales, int64_t oc, int64_t ic, void* out,
                     int out_dtype, void* stream);
/* fp3_unpack (nibble) -- 01_core/fp3_emu.py:76. */
SPARK_API int spark_fp3_unpack_nibble(const uint8_t* codes, const uint8_t* scales, int64_t oc, int64_t ic, void* out,
                            int out_dtype, void* stream);
/* fp3_fake_quant -- 01_core/fp3_emu.py:24 (FP3STE backward is the identity, :96-98). */
SPARK_API int spark_fp3_fake_quant(const void* w, int w_dtype, int64_t oc, int64_t ic, void* out, int out_dtype,
                         void* stream);

/* ---------------------------------------------------------------- NVFP4 */
/* nvfp4_pack -- 01_core/nvfp4_emu.py:81. */
SPARK_API int spark_nvfp4_pack(const void* w, int w_dtype, int64_t oc, int64_t ic, uint8_t* codes, uint8_t* scales,
                     void* stream);
/* nvfp4_unpack -- 01_core/nvfp4_emu.py:109. */
SPARK_API int spark_nvfp4_unpack(const uint8_t* codes, const uint8_t* scales, int64_t oc, int64_t ic, void* out,
                       int out_dtype, void* stream);
/* NVFP4 embedding lookup -- the forward of NVFP4EmbeddingQAT, 02_model/quant_linear.py:527-537
 * (F.embedding of the NVFP4 table), on the packed table (codes [rows, pad16(dim)/2], scales
 * [rows, pad16(dim)/16]): out[i, :] = decode(row ids[i]), int64 ids.  An id outside
 * [0, num_embeddings) gives a zero row and, when err is non-null, stores error code 7 there (pass
 * a spark_linear workspace and read it with spark_workspace_check). */
SPARK_API int spark_nvfp4_embedding(const uint8_t* codes, const uint8_t* scales, int64_t num_embeddings, int64_t dim,
                                    const int64_t* ids, int64_t n_ids, void* out, int out_dtype, int* err,
                                    void* stream);
/* Native block-scaled FP4 linear, a reported mode beside the parity path (no reference
 * counterpart; the reference quantises only weights to NVFP4, nvfp4_emu.py:37-57): the
 * activations are NVFP4 too (xq, x_scales = spark_nvfp4_pack of x [M, ic]) and
 * y[M, oc] = dequant(xq) . dequant(wq)^T runs on tcgen05.mma kind::mxf4nvf4 (block16, ue4m3
 * scales, fp32 accumulate) with both operands packed.  wq / w_scales: spark_nvfp4_pack of the
 * weight [oc, ic] (row-major codes [oc, ic/2], scales [oc, ic/16], all scales non-negative).
 * oc a multiple of 128, ic a multiple of 256, 16-byte aligned inputs; y [M, ldy] of y_dtype.  A
 * bounded in-kernel wait that expires stores error code 4 in *err (read it with
 * spark_workspace_check on a workspace whose first int is err). */
SPARK_API int spark_nvfp4_native_linear(const uint8_t* wq, const uint8_t* w_scales, const uint8_t* xq,
                                        const uint8_t* x_scales, int64_t M, int64_t oc, int64_t ic, void* y,
                                        int y_dtype, int64_t ldy, int* err, void* stream);
/* nvfp4_fake_quant -- 01_core/nvfp4_emu.py:37 (NVFP4STE backward is the identity, :66-68). */
SPARK_API int spark_nvfp4_fake_quant(const void* w, int w_dtype, int64_t oc, int64_t ic, void* out, int out_dtype,
                           void* stream);

/* ---------------------------------------------------------------- 2:4 SPFP2 */
/* two_four_pack -- 01_core/two_four.py:112.  packed: ceil(oc*ceil(ic/16)/2)*7 bytes. */
SPARK_API int spark_twofour_pack(const void* w, int w_dtype, int64_t oc, int64_t ic, uint8_t* packed, void* stream);
/* two_four_unpack -- 01_core/two_four.py:158. */
SPARK_API int spark_twofour_unpack(const uint8_t* packed, int64_t n_elements, void* out, int out_dtype, void* stream);
/* two_four_fake_quant -- 01_core/two_four.py:70 (TwoFourSTE backward is the identity, :65-67). */
SPARK_API int spark_twofour_fake_quant(const void* w, int w_dtype, int64_t n, void* out, int out_dtype, void* stream);
/* 2:4-sparse SPFP2 linear on the sparse tensor cores: y[M, oc] = x . decode(W)^T (+ bias), the
 * forward of spark_v3_twofour_forward (01_core/spark_v3_twofour.cu:124-181), W in the reference's
 * 2:4 layout (two_four_pack of [oc, ic]).  Each group of four columns holds at most two nonzeros:
 * they are kept (bf16, exact) with their positions as metadata for tcgen05.mma.sp kind::f16, so the
 * MMA skips the zero half.  x bf16 [M, ic] contiguous, 16-byte aligned; oc a multiple of 128, ic
 * of 128; y [M, ldy] of y_dtype.  An expired bounded wait stores error code 6 in *err. */
SPARK_API int spark_twofour_sparse_linear(const uint8_t* wq, const void* x, int64_t M, int64_t oc, int64_t ic,
                                          const void* bias, int bias_dtype, void* y, int y_dtype, int64_t ldy,
                                          int* err, void* stream);

/* ---------------------------------------------------------------- INT8 (lm_head tier) */
/* int8_fake_quant -- 01_core/int8_emu.py:12 (INT8STE backward is the identity, :26-27):
 * per-row symmetric, scale = max(amax/127, 1e-12), q = clamp(round(w/scale), +-127). */
SPARK_API int spark_int8_fake_quant(const void* w, int w_dtype, int64_t oc, int64_t ic, void* out, int out_dtype,
                                    void* stream);
/* ptq_int8_pack -- 01_core/int8_emu.py:37: q int8 [oc, ic], scale fp32 [oc]. */
SPARK_API int spark_int8_pack(const void* w, int w_dtype, int64_t oc, int64_t ic, int8_t* q, float* scale,
                              void* stream);
/* ptq_int8_unpack -- 01_core/int8_emu.py:49: out = q * scale[row]. */
SPARK_API int spark_int8_unpack(const int8_t* q, const float* scale, int64_t oc, int64_t ic, void* out, int out_dtype,
                                void* stream);

/* ---------------------------------------------------------------- linear */
/* y[M, oc] = x[M, ic] . decode(W)^T (+ bias), fp32 accumulation.
 * Replaces spark_v3_spfp2_linear_forward / spark_v3_spfp2_forward
 * (01_core/spark_v3_kernel.cu:172-214) and spark_v3_twofour_forward
 * (01_core/spark_v3_twofour.cu:162-181), and the decode + F.linear of the layer
 * classes (02_model/quant_linear.py:133-148, 197-212; 02_model/fp3_linear.py:46-56).
 *   fmt      SPARK_FMT_*; wq/scales in that format for a row-major [oc, ic] weight
 *            (scales NULL for SPFP2 / 2:4)
 *   x        [M, ic] with row stride ldx (elements), dtype x_dtype (bf16, f16 or f32)
 *   bias     NULL or [oc] of bias_dtype
 *   y        [M, oc] with row stride ldy, dtype y_dtype
 *   workspace  device scratch of spark_linear_workspace_size() bytes, zero-filled
 *            before its first use; calls that share a workspace must not overlap on
 *            the GPU (use one workspace per stream).
 */
SPARK_API size_t spark_linear_workspace_size(int fmt, int64_t M, int64_t oc, int64_t ic);
SPARK_API int spark_linear(int fmt, const uint8_t* wq, const uint8_t* scales, const void* x, int x_dtype, int64_t M,
                 int64_t oc, int64_t ic, int64_t ldx, const void* bias, int bias_dtype, void* y, int y_dtype,
                 int64_t ldy, void* workspace, size_t workspace_bytes, void* stream);
/* spark_linear plus an L2 prefetch hint: `prefetch_bytes` bytes at `prefetch`
 * (16-byte aligned; typically the next layer's weight) are requested into L2
 * by the decode GEMV while it runs, so the next launch finds them there.  The
 * hint changes no result; other paths ignore it.  No reference counterpart. */
SPARK_API int spark_linear_prefetch(int fmt, const uint8_t* wq, const uint8_t* scales, const void* x, int x_dtype,
                                    int64_t M, int64_t oc, int64_t ic, int64_t ldx, const void* bias, int bias_dtype,
                                    void* y, int y_dtype, int64_t ldy, void* workspace, size_t workspace_bytes,
                                    const void* prefetch, int64_t prefetch_bytes, void* stream);

/* spark_linear without a workspace argument, for callers that may not allocate
 * device memory when they run a linear (a runtime whose memory plan is fixed
 * before the first token, a C host with no device allocator).  No counterpart in
 * the reference.  Same arguments, formats and results as spark_linear (both
 * the decode GEMV and the tcgen05 GEMM routes); it allocates nothing.  Its
 * scratch is one static 16 MiB array per device inside the library, so a call
 * must fit it: spark_linear_workspace_size(fmt, M, oc, ic) <= 16 MiB, which
 * holds for every token count up to ic = 182,204 on a 148-SM GPU.  A call
 * that does not fit returns SPARK_ERR_WORKSPACE with a message naming this
 * entry point.
 *   - The first call on a device (with that device current) looks the scratch
 *     up, clears it and synchronises `stream`; make it before any stream capture
 *     (during a capture it returns SPARK_ERR_INVALID).
 *   - All calls on one device share the scratch: calls that overlap on the GPU
 *     (other streams, other threads) race, and the scratch keeps the last call's
 *     contents.  Order them on one stream.
 *   - Device-side wait expiries are recorded in the shared scratch's error word,
 *     which no entry point reads; callers that need that report use spark_linear
 *     with their own workspace and spark_workspace_check. */
SPARK_API int spark_linear_noalloc(int fmt, const uint8_t* wq, const uint8_t* scales, const void* x, int x_dtype,
                                   int64_t M, int64_t oc, int64_t ic, int64_t ldx, const void* bias, int bias_dtype,
                                   void* y, int y_dtype, int64_t ldy, void* stream);

/* EXPERIMENTAL (measured slower than the launches it replaces: 0.83 vs 0.65 ms
 * for a 14-op MLP chain at M = 1, each op paying the tcgen05 decode path's
 * critical path; spark_linear_batch on tiled weights is the fast batched form).
 * A chain of dependent decode-step ops in ONE persistent launch: dequant
 * linears (SPFP2 / FP3 / NVFP4 reference layouts, bf16 x, M <= 16 tokens) and
 * SiLU(gate) * up.  It replaces a sequence of spark_linear / spark_silu_mul
 * calls (a layer's q/k/v -> o -> gate/up -> SiLU -> down, as the reference
 * model runs them one by one); no counterpart in the reference.  dep[] names
 * the earlier ops whose output the op reads (-1: none): the op's input is
 * loaded only after they complete, while its weights stream and decode
 * earlier.  Up to 16 ops; the launch is cooperative (one CTA per SM).
 *   linear:   fmt, wq, scales, x [M, ic] (row stride ldx), oc, bias, y [M, oc]
 *             (row stride ldy, y_dtype; bf16 when a later op reads it)
 *   silu_mul: x = gate, x2 = up, y = out, all bf16 [M, ic] contiguous
 * workspace: spark_linear_chain_workspace_size(n_ops) bytes, 256-byte aligned,
 * zero before its first use; launches that share it must not overlap. */
#define SPARK_CHAIN_LINEAR 0
#define SPARK_CHAIN_SILU_MUL 1
typedef struct {
    int kind;
    int fmt;
    const uint8_t* wq;
    const uint8_t* scales;
    const void* x;
    const void* x2;
    int64_t ic, ldx, oc;
    const void* bias;
    int bias_dtype;
    void* y;
    int y_dtype;
    int64_t ldy;
    int dep[2];
} SparkChainOp;
SPARK_API size_t spark_linear_chain_workspace_size(int n_ops);
SPARK_API int spark_linear_chain(const SparkChainOp* ops, int n_ops, int64_t M, void* workspace,
                                 size_t workspace_bytes, void* stream);

/* A batch of decode-sized dequant linears (1 to 48 ops, M <= 16 tokens, bf16
 * activations) in ONE persistent launch: the batch's units (16 rows x 256
 * columns) form one sequence cut into equal contiguous ranges, one per warp
 * of the grid, and each warp streams its range from HBM through its own
 * shared-memory ring, so the weight stream has no gap at op boundaries.  Up
 * to 8 tokens the weights are decoded to f16 and the activations converted
 * once per launch to f16 with a power-of-two scale per 256-column chunk;
 * above 8 tokens, or when a chunk holds an inf or NaN, the op runs on bf16.
 * No counterpart in the reference (it runs one linear per call,
 * 01_core/spark_v3_kernel.cu:172-214); it replaces a sequence of spark_linear
 * calls, e.g. the projections of a decoder layer.  Each op is a SparkChainOp
 * of kind SPARK_CHAIN_LINEAR with fmt = SPARK_FMT_SPFP2 / FP3 / NVFP4 |
 * SPARK_LAYOUT_TILED (weights from spark_tile_weights, 16-byte aligned), optionally
 * | SPARK_EPILOGUE_SILU; x bf16 [M, ic] (16-byte aligned, ldx a multiple of 8),
 * ic a multiple of 256; y [M, oc] (oc / 2 with SiLU) of y_dtype, row stride ldy;
 * dep[] = earlier ops whose output this op reads (-1: none): the op's
 * activations are read only after those ops complete, its weights stream
 * earlier.  Results equal spark_linear's within fp32 summation order.
 * workspace: spark_linear_batch_workspace_size(ops, n_ops, M) bytes, 256-byte
 * aligned, zero-filled before its first use (it may be shared with
 * spark_linear calls on the same stream); launches that share it must not
 * overlap on the GPU.  One CTA per SM: a cooperative launch when the batch
 * has dependencies, otherwise a programmatic one (it prefetches its first
 * weights while the previous kernel of the stream finishes). */
SPARK_API size_t spark_linear_batch_workspace_size(const SparkChainOp* ops, int n_ops, int64_t M);
SPARK_API int spark_linear_batch(const SparkChainOp* ops, int n_ops, int64_t M, void* workspace,
                                 size_t workspace_bytes, void* stream);

/* spark_linear_batch with the all-reduce of one op inside the launch: op
 * ar->op is a row-parallel linear (this rank holds a slice of its input
 * features, its output is a partial sum), e.g. the down projection of a
 * tensor-parallel MLP.  Each warp that finished row groups of the op stores
 * their fp32 partials into every rank's receive buffer over peer memory, as
 * 8-byte words tagged with the call number (single 64-bit stores: no fence
 * and no flag), then waits (bounded, 2 s) until every rank's words of those
 * row groups carry this call's number, sums them in rank order 0..W-1 and
 * writes y (+ bias): every rank gets the same bits, with no separate
 * all-reduce launch.  Replaces the NCCL all-reduce after the row-parallel
 * projection.
 *   recv[r]:  rank r's receive buffer of spark_batch_ar_recv_bytes(world,
 *             M, oc) bytes, 16-byte aligned, zero before the first call
 *             (mapped into this process, e.g. spark_ipc_open);
 *   counter:  this rank's call counter, one int, zero before the first call.
 * Every rank makes the same sequence of calls (CUDA graphs included) with the
 * same op shapes; the op may not use SPARK_EPILOGUE_SILU and no other op of
 * the batch may read its output (SPARK_ERR_UNSUPPORTED); M <= 16; 1 to
 * SPARK_MAX_PEERS ranks (spark_batch_ar_recv_bytes returns 0 outside).  A
 * peer that does not arrive in 2 s sets the workspace error word
 * (spark_workspace_check).  workspace: spark_linear_batch_ar_workspace_size(
 * ops, n_ops, M, ar) bytes (ar's buffers may be null for that query). */
typedef struct {
    int op;
    int world, rank;
    void* const* recv;
    int* counter;
} SparkBatchAllReduce;
SPARK_API size_t spark_linear_batch_ar_workspace_size(const SparkChainOp* ops, int n_ops, int64_t M,
                                                      const SparkBatchAllReduce* ar);
SPARK_API int64_t spark_batch_ar_recv_bytes(int world, int64_t M, int64_t oc);
SPARK_API int spark_linear_batch_ar(const SparkChainOp* ops, int n_ops, int64_t M, const SparkBatchAllReduce* ar,
                                    void* workspace, size_t workspace_bytes, void* stream);

/* Fragment-major copy of a packed weight for spark_linear(fmt | SPARK_LAYOUT_TILED):
 * the same bytes (codes and, for FP3/NVFP4, scales) permuted so every thread of the
 * decode GEMV reads its MMA fragments with coalesced 16-byte loads.  No counterpart
 * in the reference; it is built once when a layer is loaded.  spark_tiled_bytes
 * returns the size, or 0 when the shape has no tiled layout (ic not a multiple of
 * 256, 512 for 2:4). */
SPARK_API size_t spark_tiled_bytes(int fmt, int64_t oc, int64_t ic);
SPARK_API int spark_tile_weights(int fmt, const uint8_t* wq, const uint8_t* scales, int64_t oc, int64_t ic,
                                 uint8_t* tiled, void* stream);

/* Reads (and clears) the error word a kernel leaves in `workspace` when one of its
 * bounded waits expires; synchronises `stream`.  Returns SPARK_OK or SPARK_ERR_DEVICE. */
SPARK_API int spark_workspace_check(void* workspace, void* stream);

/* Elementwise SiLU(gate) * up for the MLP between the gate/up and down projections
 * (the activation the reference model applies between its MLP linears). */
SPARK_API int spark_silu_mul(const void* gate, const void* up, void* out, int dtype, int64_t n, void* stream);

/* ---------------------------------------------------------------- peer all-reduce (tensor parallel)
 * One-shot all-reduce of the row-parallel down projection's partial sums over
 * peer memory, the NCCL all-reduce of the tensor-parallel MLP (config 4)
 * done by this library.  bufs[r] = rank r's partial (fp32 or bf16, n
 * elements, mapped into this process), flags[r] = rank r's flag array of
 * spark_peer_flags_count(world) zeroed ints; epochs = this rank's
 * spark_peer_flags_count(1) zeroed ints; err = an error word (code 5 when a peer did not arrive within 2 s).
 * Every rank issues the same sequence of calls; a rank may overwrite its
 * partial buffer only after the next call's barrier (alternate two buffers).
 * out = sum over ranks 0..world-1 in that order (fp32), identical on every rank. */
#define SPARK_MAX_PEERS 8
#define SPARK_IPC_HANDLE_BYTES 64
SPARK_API int spark_peer_flags_count(int world);
SPARK_API int spark_peer_allreduce(const void* const* bufs, int* const* flags, int world, int rank, int64_t n,
                                   int in_dtype, void* out, int out_dtype, int* epochs, int* err, void* stream);
/* Legacy CUDA IPC: handle (SPARK_IPC_HANDLE_BYTES) + offset of the allocation holding ptr;
 * open maps another process's buffer on the current device; close unmaps it. */
SPARK_API int spark_ipc_handle(const void* ptr, void* handle, int64_t* offset);
SPARK_API int spark_ipc_open(const void* handle, int64_t offset, void** ptr);
SPARK_API int spark_ipc_close(void* ptr, int64_t offset);
/* SiLU(gate) * up over [rows, cols] with gate / up rows ld_in elements apart
 * (the halves of a row-merged gate|up output) and out rows ld_out apart. */
SPARK_API int spark_silu_mul_rows(const void* gate, const void* up, int64_t ld_in, void* out, int64_t ld_out,
                                  int dtype, int64_t rows, int64_t cols, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* SPARK_B200_H */
