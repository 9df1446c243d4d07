/*
 * b200_sm100a.h -- libkernelsmith target profile for NVIDIA B200 (sm_100a).
 *
 * Plays the role of the reference's target/<profile>.h headers
 * (target/generic.h, target/x86_avx2.h): compile-time constants the C API
 * reports.  The kernels' own tiling is chosen at run time from the device's
 * SM count and shared-memory size, not from these macros.
 */
#ifndef KS_B200_TARGET_PROFILE_H
#define KS_B200_TARGET_PROFILE_H

#define KS_TARGET_NAME "b200-sm100a"
#define KS_B200_VERSION_STRING "0.1.0+sm_100a"

/* One warp: 32 f32 lanes per warp-wide instruction. */
#define KS_SIMD_WIDTH_F32 32

/* One 128-bit load; the TMA-staged kernels need 16-byte aligned rows. */
#define KS_PREFERRED_ALIGN 16

/* No quantized entry point needs caller workspace (same values as the
 * reference's generic profile, target/generic.h:91-98). */
#define KS_QUANT_DOT_I8_WORKSPACE_BYTES(K) 0u
#define KS_QUANT_MATVEC_I8_WORKSPACE_BYTES(ROWS, COLS) 0u
#define KS_QUANT_DOT_W4A8_WORKSPACE_BYTES(K, GROUP_SIZE) 0u
#define KS_QUANT_MATVEC_W4A8_WORKSPACE_BYTES(ROWS, COLS, GROUP_SIZE) 0u

#endif /* KS_B200_TARGET_PROFILE_H */
