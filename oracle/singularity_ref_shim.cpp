/*
 * Test infrastructure: builds the reference's OWN scalar reference ops
 * (Singularity/tests/test_and_bench_a5.cpp:150-293) for the host CPU so the
 * C oracle can be checked against them bit for bit.
 *
 * The reference file is compiled where it lies (include path given by
 * oracle/build_ref.sh); nothing from it is copied into this repository.  Two
 * things stand between it and an x86-64 build:
 *   - a top-level ARMv7 asm block (the callee-saved-register canary
 *     trampoline, :57-103), removed here by defining __asm__ away while the
 *     file is included;
 *   - two ARM assembly helpers the scalar refs call
 *     (singularity_memcpy_a5, singularity_f32_to_f16_row_a5), supplied below
 *     as portable C++ (byte copy; IEEE round-to-nearest-even fp16 convert,
 *     which is what VFPv4 vcvt.f16.f32 does in the default mode).
 * The test program's main() is renamed, hidden and garbage-collected, so none
 * of the ARM-only code it calls is linked.
 *
 * Output: oracle/_ref/libsingularity_ref.so exporting sref_* wrappers.
 */
#include <math.h>
#include <stddef.h>
#include <stdint.h>
#include <string.h>

#define __asm__(...)
#define main __attribute__((visibility("hidden"), unused)) singularity_a5_test_main
#include "tests/test_and_bench_a5.cpp"
#undef main
#undef __asm__

extern "C" {

void* singularity_memcpy_a5(void* dst, const void* src, size_t n) {
    return memcpy(dst, src, n);
}

static uint16_t shim_f32_to_f16(float f) {
    uint32_t x;
    memcpy(&x, &f, 4);
    const uint16_t sign = (uint16_t)((x >> 16) & 0x8000u);
    const uint32_t ax = x & 0x7FFFFFFFu;
    if (ax > 0x7F800000u) return (uint16_t)(sign | 0x7E00u | ((ax >> 13) & 0x3FFu));
    if (ax == 0x7F800000u) return (uint16_t)(sign | 0x7C00u);
    const int e = (int)(ax >> 23) - 127;
    if (e >= -14) {
        if (e > 15) return (uint16_t)(sign | 0x7C00u);
        const uint32_t m = ax & 0x7FFFFFu;
        uint32_t h = ((uint32_t)(e + 15) << 10) | (m >> 13);
        const uint32_t rem = m & 0x1FFFu;
        if (rem > 0x1000u || (rem == 0x1000u && (h & 1u))) h += 1u;
        return (uint16_t)(sign | h);
    }
    const int shift = -1 - e;
    if (shift > 25) return sign;
    const uint32_t m = (ax & 0x7FFFFFu) | 0x800000u;
    uint32_t h = m >> shift;
    const uint32_t rem = m & ((1u << shift) - 1u);
    const uint32_t half = 1u << (shift - 1);
    if (rem > half || (rem == half && (h & 1u))) h += 1u;
    return (uint16_t)(sign | h);
}

void singularity_f32_to_f16_row_a5(const float* src, uint16_t* dst, int n) {
    for (int i = 0; i < n; ++i) dst[i] = shim_f32_to_f16(src[i]);
}

__attribute__((visibility("default"))) float sref_fp16_to_fp32(uint16_t h) { return ref_fp16_to_fp32(h); }
__attribute__((visibility("default"))) uint16_t sref_fp32_to_fp16(float f) { return ref_fp32_to_fp16(f); }
__attribute__((visibility("default"))) float sref_vec_dot_q4_0_q8_0(int n, const void* x, const void* y) {
    float s = 0.0f;
    ref_vec_dot_q4_0_q8_0(n, &s, x, y);
    return s;
}
__attribute__((visibility("default"))) float sref_vec_dot_q8_0_q8_0(int n, const void* x, const void* y) {
    float s = 0.0f;
    ref_vec_dot_q8_0_q8_0(n, &s, x, y);
    return s;
}
__attribute__((visibility("default"))) void sref_quantize_row_q8_0(const float* x, void* y, int k) {
    ref_quantize_row_q8_0(x, y, k);
}
__attribute__((visibility("default"))) void sref_rmsnorm_f32(const float* x, const float* w, float* out, int n, float eps) {
    ref_rmsnorm_f32(x, w, out, n, eps);
}
__attribute__((visibility("default"))) void sref_softmax_f32(const float* x, float* out, int n) {
    ref_softmax_f32(x, out, n);
}
__attribute__((visibility("default"))) void sref_rope_f32(float* x, const float* cs, int hd, int nh) {
    ref_rope_f32(x, cs, hd, nh);
}
/* The reference test's generator (XorShift32, :362-379) and error metric
 * (rel_error, :381-388), so fuzz inputs are the reference's own. */
__attribute__((visibility("default"))) void sref_xorshift_fill(uint32_t seed, float* out, int n, uint32_t* state_out) {
    XorShift32 rng(seed);
    for (int i = 0; i < n; ++i) out[i] = rng.next_f32();
    if (state_out) *state_out = rng.state;
}
__attribute__((visibility("default"))) float sref_rel_error(float a, float b) { return rel_error(a, b); }

}  // extern "C"
