/*
 * kernelsmith/ks_common.h -- libkernelsmith common definitions (B200 build).
 *
 * Drop-in for the reference header of the same name
 * (pkp124/ulir-kernels include/kernelsmith/ks_common.h): identical version
 * macros, error codes and function signatures, so code compiled against
 * either header links against either library.
 */

#ifndef KERNELSMITH_COMMON_H
#define KERNELSMITH_COMMON_H

#include <stddef.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Library ABI version (reference ks_common.h:19-21). */
#define KS_VERSION_MAJOR 0
#define KS_VERSION_MINOR 1
#define KS_VERSION_PATCH 0

/* Return codes (reference ks_common.h:25-28).  The B200 build adds one more,
 * KS_ERR_DEVICE, in ks_b200.h; the four below keep their meaning. */
#define KS_OK 0
#define KS_ERR_INVALID_ARG (-1)
#define KS_ERR_WORKSPACE (-2)
#define KS_ERR_UNSUPPORTED (-3)

/* Name of the compiled target profile; a static string, never NULL.
 * Replaces reference ks_common.h:38 / ks_common.c:9.  The B200 build
 * returns "b200-sm100a". */
const char *ks_target_name(void);

/* f32 lanes of the target's vector unit.  Replaces reference
 * ks_common.h:45 / ks_common.c:11.  The B200 build reports the warp width,
 * 32, the number of f32 values one warp-wide instruction processes. */
size_t ks_simd_width_f32(void);

#ifdef __cplusplus
}
#endif

#endif /* KERNELSMITH_COMMON_H */
