// Nested metric alignment of DA3 (anyview branch + metric branch -> metric-scale depth),
// host code over the two branches' outputs; same steps, thresholds and accumulation
// types as NestedAligner (src/nested.cpp:7-96).
#pragma once
#include <stddef.h>

namespace da3b {

// torch.quantile with linear interpolation over n values (src/nested.cpp:7-20): the
// floor / ceil order statistics of position q*(n-1), found by selection (the same two
// values a full sort yields), interpolated in double. v is reordered; 0 for n == 0.
float quantile_linear(float* v, size_t n, float q);

// Mono / metric sky fill (src/nested.cpp:22-33): pixels with sky >= 0.3 take the 0.99
// quantile of the non-sky depth; a no-op unless both sets exceed 10 pixels.
void mono_sky_fill(float* depth, const float* sky, size_t n);

// Alignment (src/nested.cpp:35-96). Inputs: anyview depth / confidence [n], its
// extrinsics (3x4) and intrinsics (3x3) row-major; metric depth (after the sky fill)
// and sky [n]. Outputs: out_depth [n] (may alias any_depth) and out_ext (translation
// scaled). Returns the scale factor.
float nested_align(const float* any_depth, const float* any_conf, const float any_ext[12], const float any_intr[9],
                   const float* metric_depth, const float* sky, size_t n, float* out_depth, float out_ext[12]);

}  // namespace da3b
