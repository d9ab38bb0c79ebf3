/* Test infrastructure only: nothing under mxwave_b200/ links or runs this.
 *
 * Exhaustive CPU check of the division-free exponents the quantize kernel
 * uses (floor_log2_div6 / ceil_log2_div6 in mxwave_b200/csrc/quantize.cu)
 * against their definition, the reference's
 *   floor(torch.log2(block_max / 6.0)) and ceil(torch.log2(actual_max / 6.0))
 * (mxwave/core.py:199-206) evaluated on the fp32 quotient.
 *
 * The kernel derives the exponent from the input's own bits: with x = m*2^E,
 * fl(x/6) lies in [2^(E-2), 2^(E-1)) for m >= 1.5 and in (2^(E-3), 2^(E-2))
 * below.  torch's fp32 log2 can only round onto an integer when the quotient
 * is within 256 ulps of a power of two; the kernel sends those inputs (m just
 * under 1.5 for floor, just over it for ceil) to the division and an exact
 * log2 test.  This program checks, for every fp32 x in the kernel's domain
 * (x >= 1e-6 for floor, x >= 1e-12 for ceil), that
 *   - outside those bands the quotient is never within 256 ulps of a power
 *     of two (so the definition reduces to exponent arithmetic), and
 *   - the kernel's formula equals the exponent of the correctly rounded
 *     quotient there.
 * Exit status 0 when every value agrees.  Runs in seconds. */
#include <stdint.h>
#include <stdio.h>
#include <string.h>

static float from_bits(uint32_t b) { float x; memcpy(&x, &b, 4); return x; }
static uint32_t to_bits(float x) { uint32_t b; memcpy(&b, &x, 4); return b; }

int main(void) {
  uint64_t checked = 0, in_band = 0, bad = 0;
  const uint32_t lo = to_bits(1e-12f), hi = to_bits(3.4028235e38f);
  for (uint64_t b = lo; b <= hi; ++b) {
    const float x = from_bits((uint32_t)b);
    const float q = x / 6.0f;
    const uint32_t qb = to_bits(q);
    const int eq = (int)((qb >> 23) & 0xff) - 127;
    const uint32_t mq = qb & 0x7fffffu;
    const int E = (int)((b >> 23) & 0xff) - 127;
    const uint32_t man = (uint32_t)b & 0x7fffffu;
    if (x >= 1e-6f) { /* floor */
      const int band = man - (0x400000u - 256u) < 256u;
      if (band) {
        in_band++;
      } else {
        const int kernel = E - (man >= 0x400000u ? 2 : 3);
        if (mq >= 0x7fff00u || kernel != eq) {
          if (bad < 10) printf("floor: x=%a kernel %d quotient exponent %d\n", x, kernel, eq);
          bad++;
        }
        checked++;
      }
    }
    { /* ceil */
      const int band = man - 0x400001u < 512u;
      if (band) {
        in_band++;
      } else {
        const int kernel = E - (man > 0x400000u ? 1 : 2);
        const int def = mq == 0 ? eq : eq + 1;
        if ((mq != 0 && mq < 0x100u) || kernel != def) {
          if (bad < 10) printf("ceil: x=%a kernel %d definition %d\n", x, kernel, def);
          bad++;
        }
        checked++;
      }
    }
  }
  printf("checked %llu values (%llu in the exact-test bands), %llu disagreements\n",
         (unsigned long long)checked, (unsigned long long)in_band, (unsigned long long)bad);
  return bad != 0;
}
