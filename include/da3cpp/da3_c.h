/*
 * da3_c.h — C ABI of libda3b with the names and signatures of DA3cpplib's C API
 * (include/da3cpp/da3_c.h in DA3cpplib, :11-38; implementation src/da_capi.cpp).
 * Outputs are malloc'd and released with da_capi_free_floats / _bytes / _string;
 * failures return NULL or -1 and set da_capi_last_error (src/da_capi.cpp:97-176).
 *
 * Camera pose (camera-token decoder), nested metric models (da_capi_load_nested) and
 * DA3 mono sky planes are implemented. Point clouds and the GLB / COLMAP exporters lie
 * outside the depth path: they are exported for link compatibility and fail with a
 * last_error that says so.
 */
#ifndef DA3CPP_DA3_C_H
#define DA3CPP_DA3_C_H

#include <stddef.h>

#ifdef __cplusplus
extern "C" {
#endif

#if defined(__GNUC__)
#define DA_CAPI __attribute__((visibility("default")))
#else
#define DA_CAPI
#endif

typedef struct da_ctx da_ctx;

/* ABI version: 4, as the reference (src/da_capi.cpp:71). */
DA_CAPI int da_capi_abi_version(void);
/* Loads a GGUF onto CUDA device $DA3B_DEVICE (default 0); n_threads is accepted and unused. */
DA_CAPI da_ctx* da_capi_load(const char* gguf_path, int n_threads);
DA_CAPI da_ctx* da_capi_load_nested(const char* anyview_gguf, const char* metric_gguf, int n_threads);
DA_CAPI void da_capi_free(da_ctx* ctx);
DA_CAPI char* da_capi_info_json(da_ctx* ctx);
DA_CAPI void da_capi_free_string(char* value);
DA_CAPI const char* da_capi_last_error(da_ctx* ctx);

/* Depth of one image file (binary PPM, P6) at the processed resolution. */
DA_CAPI float* da_capi_depth_path(da_ctx* ctx, const char* image_path, int* out_h, int* out_w);
DA_CAPI int da_capi_pose_path(da_ctx* ctx, const char* image_path, float out_ext[12], float out_intr[9]);
/* Multi-view depth: all views share global attention (DA3). Returns n * h * w floats in
 * the input view order. When out_ext / out_intr are non-NULL they receive n * 12 and
 * n * 9 floats: each view's camera-to-world extrinsics and intrinsics from the camera
 * token decoder (fails, returning NULL, when the model has no camera decoder). */
DA_CAPI float* da_capi_depth_pose_multi(da_ctx* ctx, const char** image_paths, int n_images, int* out_h,
                                        int* out_w, int* out_n, float* out_ext, float* out_intr);
DA_CAPI int da_capi_depth_dense(da_ctx* ctx, const char* image_path, int* out_h, int* out_w, float** out_depth,
                                float** out_conf, float** out_sky, float out_ext[12], float out_intr[9],
                                int* out_is_metric);
DA_CAPI int da_capi_points(da_ctx* ctx, const char* image_path, float conf_thresh, int* out_n, float** out_xyz,
                           unsigned char** out_rgb);
DA_CAPI int da_capi_export_glb(da_ctx* ctx, const char* image_path, const char* out_glb);
DA_CAPI int da_capi_export_colmap(da_ctx* ctx, const char* image_path, const char* out_dir, int binary);

DA_CAPI void da_capi_free_floats(float* value);
DA_CAPI void da_capi_free_bytes(unsigned char* value);

#ifdef __cplusplus
}
#endif
#endif
