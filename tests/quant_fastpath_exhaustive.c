/* Exhaustive check of the fast int8 quantiser used by pool_quant_kernel
 * (cast_b200/csrc/select_quant.cuh, quant8_fast) against the defined one.
 *
 * Defined quantiser: s = RN(amax / 127), code = clamp(rint_half_even(RN(x / s)),
 * -127, 127) with IEEE division.  Fast path (blocks with amax >= 2^-90):
 * inv = RN(1 / s), q0 = RN(x * inv), r = fma(-q0, s, x), q1 = fma(r, inv, q0),
 * code = low byte of the bits of RN(q1 + 1.5 * 2^23).  For every positive
 * finite bf16 amax and every bf16 x with |x| <= amax the two codes must agree
 * and the fast code must not leave [-127, 127] (so the kernel needs no clamp).
 * Blocks with amax < 2^-90 use the IEEE division in the kernel too.
 * Prints "mismatches 0" and exits 0 on success. */
#include <math.h>
#include <stdint.h>
#include <stdio.h>
#include <string.h>

static float bf16_value(uint16_t h) {
  uint32_t u = (uint32_t)h << 16;
  float f;
  memcpy(&f, &u, 4);
  return f;
}
static uint32_t float_bits(float f) {
  uint32_t u;
  memcpy(&u, &f, 4);
  return u;
}

int main(void) {
  long long checked = 0, bad = 0, over = 0;
  for (uint32_t ha = 1; ha < 0x7F80; ++ha) { /* positive finite bf16, subnormals included */
    const float amax = bf16_value((uint16_t)ha);
    const float s = amax / 127.0f;
    if (!(s > 0.0f)) continue;
    const float inv = 1.0f / s;
    if (isinf(inv)) continue;
    const int exact_div = amax < 0x1p-90f;
    for (uint32_t hx = 0; hx < 0x10000; ++hx) {
      const float x = bf16_value((uint16_t)hx);
      if (!(fabsf(x) <= amax)) continue;
      const float q = x / s;
      int ref = (int)rintf(q);
      if (ref > 127) ref = 127;
      if (ref < -127) ref = -127;
      const float q0 = x * inv;
      const float r = fmaf(-q0, s, x);
      const float q1 = fmaf(r, inv, q0);
      const float t = (exact_div ? q : q1) + 12582912.0f;
      const int code = (int)(int8_t)(float_bits(t) & 0xFFu);
      const int full = (int)float_bits(t) - 0x4B400000;
      if (full > 127 || full < -127) ++over;
      if (code != ref) {
        if (bad < 10) printf("mismatch amax=%a x=%a ref=%d fast=%d\n", amax, x, ref, code);
        ++bad;
      }
      ++checked;
    }
  }
  printf("checked %lld pairs, mismatches %lld, out of range %lld\n", checked, bad, over);
  return (bad != 0 || over != 0) ? 1 : 0;
}
