/*
 * da3b.h — kernel-level C ABI of libda3b (B200 / sm_100a).
 *
 * These entry points are the drop-in replacement for the reference's GPU plugin
 * point: in DA3cpplib every hot op of the depth path is a ggml graph node
 * (ggml_mul_mat for the Q8_0 linears, ggml_flash_attn_ext, ggml_conv_2d /
 * ggml_conv_transpose_2d_p0 / ggml_interpolate for the DPT head), and its own
 * CUDA kernels enter ggml through a GGML_OP_CUSTOM descriptor
 * {magic, launch(dst, stream, user), user}
 * (scripts/patches/ggml/0001-da3-custom-cuda-ops.patch:24-38,
 *  src/cuda_head_kernels.hpp:28-49, src/cuda_head_kernels.cu:20-25).
 * Here each op is a flat extern "C" function taking raw device pointers, sizes
 * and a cudaStream_t (passed as void*), returning 0 on success or a negative
 * error code. No function allocates on the caller's behalf except where stated.
 *
 * Layouts: activations are row-major f16 ([rows][cols], cols fastest) or NHWC
 * f16 ([B][H][W][C]); weights are f16 [N][K] (K fastest); biases are f32.
 */
#ifndef DA3B_H
#define DA3B_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#if defined(__GNUC__)
#define DA3B_API __attribute__((visibility("default")))
#else
#define DA3B_API
#endif

/* Version of this kernel-level ABI. */
DA3B_API int da3b_abi_version(void);

/* Waits for the current device, then returns (and clears) the device-side status
 * word that bounded waits inside the kernels write on a timeout (0 = ok). Returns
 * a negative value if the device itself reports an error. */
DA3B_API int da3b_device_status(void);

/* Q8_0 weight repack: GGUF Q8_0 rows (K/32 blocks of {f16 d, int8 q[32]}) on the
 * device -> f16 plane w[r][k] = d*q with leading dimension ldw (>= K, multiple of
 * 32, zero padded). Replaces the per-call Q8_0 dequantisation inside ggml_mul_mat
 * (src/ggml_extend.hpp:6-10) by a load-time repack. */
DA3B_API int da3b_dequant_q8_0(const void* q8, int rows, int K, void* w_f16, int ldw, void* stream);

/* Linear layer y = act(x W^T + b) (+res): the replacement of `linear()`
 * (src/ggml_extend.hpp:6-10 -> ggml_mul_mat(W_q8_0, x) + bias) on the tcgen05 path.
 * x: f16 [M][K] (lda), W: f16 [N][K] (ldw, from da3b_dequant_q8_0), bias f32 [N]
 * or NULL, act: 0 none, 1 relu, 2 erf-GELU (src/ggml_extend.hpp:22-25), 3 the same GELU
 * with a one-reciprocal erf approximation (Abramowitz & Stegun 7.1.28),
 * out: f16 [M][N] (ldo). */
DA3B_API int da3b_linear_f16(const void* x, int M, int K, int lda, const void* w, int N, int ldw,
                             const float* bias, int act, void* out, int ldo, void* stream);

/* Residual linear: resid[m][n] += scale[n] * ((x W^T)[m][n] + bias[n]) in f32 —
 * the ViT block's `x + ls * linear(...)` (src/vit_block.cpp:33-35, :56-57).
 * scale may be NULL (no LayerScale). */
DA3B_API int da3b_linear_resid_f32(const void* x, int M, int K, int lda, const void* w, int N, int ldw,
                                   const float* bias, const float* scale, float* resid, int ldr, void* stream);

/* Planar Q8_0, the resident form of the ViT block linears: the GGUF Q8_0 bytes of W
 * [N][K] (K % 32 == 0, N % 8 == 0) as an int8 plane q [N][K] followed by the f16 block
 * scales transposed, d [K/32][N] (the same byte count, rows a TMA can tile).
 *   da3b_repack_q8_0_planar: GGUF Q8_0 rows on the device -> planar Q8_0.
 *   da3b_dequant_q8p:        planar Q8_0 -> f16 w [N][K] = f16(d * q), bit-identical
 *                            to da3b_dequant_q8_0.
 *   da3b_linear_q8p_f16 / da3b_linear_q8p_resid_f32: da3b_linear_f16 /
 *                            da3b_linear_resid_f32 with W planar Q8_0, the weight tiles
 *                            dequantised in shared memory by the GEMM (the dequantisation
 *                            inside ggml_mul_mat(W_q8_0, x), src/ggml_extend.hpp:6-10);
 *                            bit-identical to the f16 route on da3b_dequant_q8p's
 *                            weights. They serve the one-CTA tile regime (few rows, e.g.
 *                            one image's 1370 tokens) and return 1 without launching
 *                            when M x N is a problem for the CTA-pair kernel. */
DA3B_API int da3b_repack_q8_0_planar(const void* q8, int N, int K, void* planar, void* stream);
DA3B_API int da3b_dequant_q8p(const void* planar, int N, int K, void* w_f16, void* stream);
DA3B_API int da3b_linear_q8p_f16(const void* x, int M, int K, int lda, const void* planar, int N,
                                 const float* bias, int act, void* out, int ldo, void* stream);
DA3B_API int da3b_linear_q8p_resid_f32(const void* x, int M, int K, int lda, const void* planar, int N,
                                       const float* bias, const float* scale, float* resid, int ldr, void* stream);

/* Bidirectional attention softmax(q k^T / 8) v over head_dim 64 — the replacement of
 * ggml_flash_attn_ext with F32 precision in attention() (src/attention.cpp:44-96).
 * qkv: f16 [nseq*seqlen][3*heads*64] (q | k | v, head h at columns h*64 of each third,
 * the layout of the QKV linear's output), out: f16 [nseq*seqlen][heads*64]. */
DA3B_API int da3b_attention(const void* qkv, int nseq, int seqlen, int heads, void* out, void* stream);

/* Q8_0 x Q8_0 linear on the int8 tensor cores (tcgen05.mma kind::i8), bit-exact with the
 * reference's CPU ggml_mul_mat(W_q8_0, x) (src/ggml_extend.hpp:6-10): x quantised per
 * 32-element block (da3b_quantize_q8_0), exact int32 block dot products, and
 * y[m][n] = sum over blocks b in order of float(isum_b) * (d_w * d_x) (+ bias[n]) in
 * explicitly rounded f32. The product path uses the f16 GEMM (da3b_linear_f16); this
 * entry point is the measured int8 route and a reference-exact linear.
 *   da3b_quantize_q8_0: x f32 [M][K] -> q int8 [M][K], d f32 [M][K/32] (the f16 scale).
 *   da3b_repack_q8_0:   GGUF Q8_0 rows [N][K/32][34 B] -> qw int8 [N][K] and the scales
 *                       transposed, dw_t f32 [K/32][N].
 *   da3b_linear_q8q8_i8: K % 128 == 0, N % 128 == 0, y f32 [M][ldy] (16-byte aligned,
 *                       ldy % 4 == 0), bias f32 [N] or NULL. */
DA3B_API int da3b_quantize_q8_0(const float* x, int M, int K, void* q_int8, float* d, void* stream);
DA3B_API int da3b_repack_q8_0(const void* q8, int N, int K, void* qw_int8, float* dw_t, void* stream);
DA3B_API int da3b_linear_q8q8_i8(const void* qx, const float* dx, int M, int K, const void* qw, const float* dw_t,
                                 int N, const float* bias, float* y, int ldy, void* stream);

/* Wait-timeout probe (tests of the failure path every pipelined kernel shares): one
 * CTA waits, through the kernels' bounded mbarrier wait, on a barrier that nothing
 * arrives on, with a limit of limit_ns (1 ns .. 1 s) instead of the kernels' 2 s.
 * The wait runs out, the status word becomes 1 (a timed-out wait), and the kernel
 * returns; with use_tmem it first allocates tensor memory and frees it after the
 * failed wait, the way the kernels do. status_dev = NULL uses the library's status
 * word (read and cleared by da3b_device_status); elapsed_dev (may be NULL) receives
 * the nanoseconds waited. No GPU fault is involved: the context stays usable. */
DA3B_API int da3b_debug_wait_timeout(unsigned long long limit_ns, int use_tmem, int* status_dev,
                                     unsigned long long* elapsed_dev, void* stream);

/* Tensor-pipe rate probe (no counterpart in the reference; measurement only): ctas CTAs
 * of one per SM each issue iters x 4 back-to-back tcgen05.mma of M = 128, K = 16, N = n
 * (64, 80, 128 or 256) f16 into one TMEM accumulator, A from shared memory
 * or (a_tmem != 0) tensor memory, and write the cycles from the first issue to the
 * completion of the last to cycles_dev[cta] (u64; 0 if a bounded wait gave up). */
DA3B_API int da3b_debug_mma_cycles(int n, int a_tmem, int iters, int ctas, unsigned long long* cycles_dev,
                                   void* stream);

/* Key-range split of the flash attention (process-wide): n < 0 automatic (default: when
 * the (query tile, head, sequence) grid would leave SMs idle, each query tile's keys are
 * shared out over a cluster of up to 4 CTAs, at least 6 key tiles each, which merge their
 * partial softmax sums); n = 0 or 1 never; n = 2..4 that many shares wherever the
 * sequence has that many 64-key tiles. For tests and measurement; returns 0. */
DA3B_API int da3b_set_attention_split(int n);

/* The tiles da3b_linear_f16 / da3b_linear_resid_f32 choose for an M x N x K linear (host
 * only, no GPU work): returns 1 for the one-CTA kernel with tile width *bn and K split
 * *ksplit (a cluster of that many CTAs per tile), 0 for CTA pairs of tile width *bn,
 * negative for bad arguments. The one-CTA choice comes from a cost model fitted to B200
 * timings at a few images' rows (one ViT-B image: QKV and fc1 on 256-wide tiles, fc2 on
 * 128-wide tiles split in two, attn proj on 64-wide tiles). */
DA3B_API int da3b_linear_tiles(int M, int N, int K, int* bn, int* ksplit);

/* The two halves of da3b_attention, for callers that keep V transposed (the engine's
 * QKV GEMM epilogue writes it that way): da3b_transpose_v writes V^T f16
 * [nseq][heads][64][ld_vt] (ld_vt >= seqlen, a multiple of 8; columns beyond seqlen are
 * never read), and da3b_attention_vt runs the flash-attention kernel alone on q, k from
 * qkv and that V^T. Same arithmetic as da3b_attention. */
DA3B_API int da3b_transpose_v(const void* qkv, int nseq, int seqlen, int heads, void* vt, int ld_vt, void* stream);
DA3B_API int da3b_attention_vt(const void* qkv, const void* vt, int ld_vt, int nseq, int seqlen, int heads, void* out,
                               void* stream);

/* Capacity of the fixed V^T scratch of da3b_attention_noalloc, in bytes (32 MiB):
 * nseq * heads*64 * round_up(seqlen, 8) * 2 must not exceed it, e.g. 11 ViT-L images
 * of 1370 tokens, or one 8-view scene of 1297 tokens per view at 16 heads. */
#define DA3B_NOALLOC_VT_BYTES (32u << 20)
/* Returned by da3b_attention_noalloc when a call needs more than DA3B_NOALLOC_VT_BYTES
 * of scratch; nothing is launched. Split the batch (fewer sequences per call). */
#define DA3B_ERR_NOALLOC_TOO_LARGE (-103)

/* da3b_attention without any device allocation by the library. It has no counterpart
 * in the reference (DA3cpplib's attention runs inside a ggml graph whose allocator
 * owns all memory); it exists for callers that cannot let a library allocate device
 * memory on their call path, for example a host under a fixed device-memory budget
 * or with its own allocator owning the device, or a latency-critical loop that cannot
 * take cudaMalloc's implicit device synchronisation on a first or larger call.
 * Same inputs, outputs and arithmetic as da3b_attention (bit-identical results); the
 * differences:
 *  - the V^T scratch is a fixed file-scope device array of DA3B_NOALLOC_VT_BYTES per
 *    device, created with the library's module; larger calls are rejected with
 *    DA3B_ERR_NOALLOC_TOO_LARGE before anything is launched;
 *  - the first call on each device resolves that array's address
 *    (cudaGetSymbolAddress); make that first call before capturing the stream;
 *  - the caller owns the status word: status_dev points to a device int that must
 *    start at zero and that a timed-out wait inside the kernel sets non-zero (the
 *    library never clears it); the scratch itself needs no initial value;
 *  - there is ONE scratch per device: calls that overlap in time on the same device
 *    (different streams, or threads without ordering) race on it and corrupt each
 *    other's results. Order them on one stream, or synchronise between them.
 * Returns 0 when launched, a negative code otherwise. */
DA3B_API int da3b_attention_noalloc(const void* qkv, int nseq, int seqlen, int heads, void* out, int* status_dev,
                                    void* stream);

/* Packs a ggml conv2d weight (ne [KW,KH,IC,OC] f32 == torch [OC][IC][KH][KW]) into
 * the implicit-GEMM layout f16 [OC][KH*KW][icp], icp = IC rounded up to 64. */
DA3B_API int da3b_pack_conv_weight(const float* w_f32, int OC, int IC, int ksize, void* w_packed, void* stream);

/* KxK stride-1 "same" convolution (K = 1 or 3) on NHWC f16, implicit GEMM:
 *   v = conv(x, w) + bias + res1 + res2;  out = act(v);  out_relu = relu(v) (optional)
 * Replaces conv2d / residual_conv_unit pieces of src/dpt_blocks.cpp:18-114 and the
 * fused kernels k_conv3x3_igemm / k_conv1x1_igemm (src/cuda_head_kernels.cu:34-164).
 * x: [B][H][W][IC], w: packed (da3b_pack_conv_weight), res1/res2/out/out_relu:
 * [B][H][W][OC] or NULL. */
DA3B_API int da3b_conv_nhwc(const void* x, int B, int H, int W, int IC, const void* w_packed, int OC,
                            int ksize, const float* bias, const void* res1, const void* res2, int act,
                            void* out, void* out_relu, void* stream);

/* Align-corners bilinear resize of NHWC f16 [B][hs][ws][C] to [B][H][W][C] (C a
 * multiple of 8), the DPT head's upsample: interp_bilinear_ac (src/dpt_blocks.cpp:87-90,
 * ggml_interpolate with GGML_SCALE_FLAG_ALIGN_CORNERS). */
DA3B_API int da3b_upsample_nhwc(const void* in, int B, int hs, int ws, int C, void* out, int H, int W, void* stream);

/* DPT output stage: output_conv2 on the align-corners upsample of out1, fused: feat NHWC
 * f16 [B][hs][ws][C] (C a multiple of 16, at most 128) is upsampled to H x W (+ pe, NHWC
 * f16 [H][W][C] or NULL: the 0.1 UV embedding of head_pos_embed), then the 3x3 conv
 * (da3b_pack_conv_weight layout, 32 output channels, out2a_bias) -> relu -> 1x1 conv
 * out2b_w [od][32] + out2b_b -> act[o] per output channel (0 identity, 1 relu, 2
 * sigmoid * scale, 3 exp, 4 exp + 1) into out[o], f32 [B][H][W] device planes (od <= 8).
 * Replaces interp_bilinear_ac + add_uv_input + the out2a / out2b convs of
 * DptHead::build_depth_graph (src/dpt_head.cpp:199-222) and the activations of
 * src/dpt_head.cpp:327-338 / :402-439. fused = 0 runs the same through a materialised
 * f16 upsampled map (da3b_upsample_nhwc + the conv), for comparison. */
DA3B_API int da3b_output_conv2(const void* feat, int B, int hs, int ws, int C, const void* pe, int H, int W,
                               const void* w_packed, const float* out2a_bias, const float* out2b_w,
                               const float* out2b_b, int od, const int* act, float scale, float* const* out,
                               int fused, void* stream);

/* uint8 HWC RGB resize of B images [B][sh][sw][3] -> [B][dh][dw][3], bit-exact with
 * DA3cpplib's resizers: mode 0 = resize_cubic (src/preprocess.cpp:61-99), mode 1 =
 * resize_area (:122-148, which falls back to its bilinear when both axes grow). src and
 * dst are device memory. The library keeps per-size tap tables and a float scratch per
 * device, allocated on first use of a size. */
DA3B_API int da3b_resize_u8(const void* src, int B, int sw, int sh, void* dst, int dw, int dh, int mode, void* stream);

/* Legacy preprocess of B RGB8 images [B][h][w][3] (device): the reference's float
 * bilinear resize to the floor-to-patch size and normalisation (src/preprocess.cpp:8-41),
 * bit-exact, into planar f32 [B][3][*out_h][*out_w] (device; NULL: size query only).
 * mean/std are host arrays of 3. */
DA3B_API int da3b_preprocess_legacy(const void* rgb, int B, int w, int h, int patch, const float* mean,
                                    const float* std_, void* chw_out, int* out_h, int* out_w, void* stream);

/* Normalise + patchify: RGB8 [B][H][W][3] (device, H and W multiples of patch) ->
 * the patch-embed GEMM operand f16 [B*(H/patch)*(W/patch)][ldk], column
 * c*patch^2 + ky*patch + kx = (v/255 - mean[c]) / std[c] (src/preprocess.cpp:192-196),
 * zero up to ldk (even, >= 3*patch^2). mean/std are host arrays of 3. */
DA3B_API int da3b_patchify(const void* rgb, int B, int H, int W, int patch, const float* mean, const float* std_,
                           void* out, int ldk, void* stream);

/* ======================================================================
 * Model-level entry points (batched depth path). A context is the same
 * da_ctx as the reference-compatible C ABI in da3cpp/da3_c.h.
 * ====================================================================== */
typedef struct da_ctx da_ctx;

/* Loads a GGUF (DA3cpplib weight layout) onto CUDA device `device`: the
 * replacement of Engine::load + ModelLoader::offload_weights
 * (src/engine.cpp:24-66, src/model_loader.cpp:166-220). NULL on failure. */
DA3B_API da_ctx* da3b_load(const char* gguf_path, int device);

/* Processed size of a w x h input under the reference preprocessing policy
 * (preprocess_real, src/preprocess.cpp:157-197; legacy=1: floor-to-patch,
 * src/preprocess.cpp:26-41). *needs_resize = 1 when the image must be resampled. */
DA3B_API int da3b_processed_size(da_ctx* ctx, int w, int h, int legacy, int* out_h, int* out_w, int* needs_resize);

/* Depth of n_views RGB8 images [n_views][h][w][3] (device memory), h and w at the
 * processed size. views_per_scene consecutive views share global attention (1 =
 * independent images, the path of Engine::depth_native_fused / depth_relative,
 * src/engine.cpp:121-130, :189-229; > 1 = Engine::depth_pose_multi's backbone,
 * src/engine.cpp:352-384). Outputs (device memory, f32): depth [n][h][w], conf
 * [n][h][w] (DA3 only, may be NULL), rays [7][n][8h/14][8w/14] (aux ray head, may
 * be NULL). Asynchronous on `stream` after the first call of a shape. */
DA3B_API int da3b_infer_device(da_ctx* ctx, const void* rgb_dev, int n_views, int views_per_scene, int h, int w,
                               void* depth_dev, void* conf_dev, void* rays_dev, void* stream);

/* Same with host buffers (copies included); returns after the results are on the host. */
DA3B_API int da3b_infer_host(da_ctx* ctx, const void* rgb_host, int n_views, int views_per_scene, int h, int w,
                             float* depth_host, float* conf_host, float* rays_host);

/* Depth from n_views already preprocessed images: normalised planar f32
 * [n_views][3][h][w] (host or device memory, h and w multiples of the patch size), the
 * input of infer_preprocessed (src/api.cpp:178-193, Engine::depth_native_prepared at
 * src/engine.cpp:230-270) without the callback. depth / conf as in da3b_infer_device
 * (host or device). Asynchronous on `stream` (NULL: the context's stream) after the first
 * call of a shape. */
DA3B_API int da3b_infer_prepared(da_ctx* ctx, const float* chw, int n_views, int h, int w, float* depth, float* conf,
                                 void* stream);

/* Camera pose of the n_views views of the last run (DA3 checkpoints with a camera
 * decoder, cam.*): the camera-token MLP of CamPose::pose (src/cam_pose.cpp:8-83) on the
 * out-layer-3 camera tokens, in the original view order. pose_enc [n][9] = t(3),
 * quaternion xyzw (4), fov h/w (2); ext [n][12] world-to-camera 3x4; intr [n][9].
 * Host arrays, each may be NULL. */
DA3B_API int da3b_last_pose(da_ctx* ctx, int n_views, float* pose_enc, float* ext, float* intr);

/* Ray -> pose solver (use_ray_pose: solve_ray_pose at src/ray_pose.cpp:95-252 with its
 * production defaults, as Engine::depth_pose_rays_native runs it, src/engine.cpp:296-328)
 * on view `view` of a device ray field rays_dev [7][n_views][ray_h][ray_w] f32 (direction
 * xyz, origin xyz, confidence; the layout da3b_infer_device's rays output has). ext [12]
 * camera-to-world 3x4 and intr [9] (host), for an image of img_h x img_w; diag (host, 26
 * doubles, may be NULL) = R (9), T (3), focal (2), pp (2), refit homography (9), best
 * inlier count. Returns 0, 1 for a degenerate field (the reference's false), or a negative
 * error. Synchronises the stream (NULL: the context's). */
DA3B_API int da3b_ray_pose(da_ctx* ctx, const float* rays_dev, int n_views, int view, int ray_h, int ray_w,
                           int img_h, int img_w, float* ext, float* intr, double* diag, void* stream);

/* Sky plane of the last run of a model with a sky head (DA3 mono / metric DPT,
 * head.scratch.sky_out2a / sky_out2b; DptHead::depth_sky at src/dpt_head.cpp:396-400 with
 * the relu of src/dpt_head.cpp:334-338): sky [n_views][H][W] host array. */
DA3B_API int da3b_last_sky(da_ctx* ctx, int n_views, float* sky);

/* Nested metric alignment on host arrays of n pixels (NestedAligner::process_mono_sky and
 * ::align, src/nested.cpp:22-96, as Engine::depth_metric runs them at
 * src/engine.cpp:446-449): metric_depth is sky-filled in place first; out_depth [n] and
 * out_ext [12] receive the aligned depth and the translation-scaled anyview extrinsics.
 * Returns the scale factor (negative on bad arguments). No GPU work. */
DA3B_API float da3b_nested_align(const float* any_depth, const float* any_conf, const float* any_ext,
                                 const float* any_intr, float* metric_depth, const float* sky, int64_t n,
                                 float* out_depth, float* out_ext);

/* Reference view chosen per scene by the last multi-view run (views_per_scene >= 3). */
DA3B_API int da3b_ref_views(da_ctx* ctx, int* out, int n);
/* Kernel launches of one forward of that shape (after one run of it). */
DA3B_API int da3b_launches(da_ctx* ctx, int n_views, int views_per_scene, int h, int w, int rays);
/* Out-layer feature map of the last run (f16 [rows][cols], token 0 dropped) copied to host. */
DA3B_API int da3b_debug_feature(da_ctx* ctx, int layer, void* out_f16, size_t capacity, int* rows, int* cols);
/* 1 = every later forward also keeps the residual stream after each ViT block (f32
 * [depth][rows][embed_dim] on the device, rows = views x tokens in processing order);
 * 0 = off (default). Changing it drops the cached plans. For per-layer parity tests. */
DA3B_API int da3b_set_capture_residuals(da_ctx* ctx, int on);
/* Residual stream after block `layer` of the last run (f32 [rows][cols]) copied to
 * host; -2 when residual capture was off for that run. */
DA3B_API int da3b_debug_residual(da_ctx* ctx, int layer, float* out_f32, size_t capacity, int* rows, int* cols);
/* 1 = replay captured CUDA graphs (default), 0 = eager launches. */
DA3B_API int da3b_set_graphs(da_ctx* ctx, int on);
/* 1 = activations entering each Q8_0 linear are rounded through Q8_0 the way ggml
 * quantises them before its Q8_0 x Q8_0 dot products (ggml_mul_mat,
 * src/ggml_extend.hpp:6-10); 0 (default) = plain f16 activations, which stay closer
 * to the reference's outputs than a second, independent Q8_0 rounding does. */
DA3B_API int da3b_set_act_quant(da_ctx* ctx, int on);
/* 1 = the depth / confidence / ray outputs are the raw head logits (no output
 * activation), for parity checks against pre-activation reference values. */
DA3B_API int da3b_set_raw_logits(da_ctx* ctx, int on);
/* out[10] = {embed_dim, depth, num_heads, patch_size, cat_token, output_dim, has_aux, is_da2,
 *            has_sky, has_camera} */
DA3B_API int da3b_model_dims(da_ctx* ctx, int* out);

#ifdef __cplusplus
}
#endif

#endif /* DA3B_H */
