// rope_table.cpp — host side of the rotary embedding: the angle, cosine and
// sine of every (position, pair) with exactly the single-precision operations
// of ops::rope (src/cpu/ops.rs:429-432): e = (2 * i) / dim, p = theta^e
// (powf), angle = position / p, then sinf / cosf of the angle.  The device
// kernel only rotates with these values, so the rotation matches the
// reference bit for bit on a host whose C library the reference also uses.
#include <math.h>

#include "kernels.h"

namespace uocr {

void build_rope_table(int dim, float theta, int max_pos, float* cos_sin) {
  const int half = dim / 2;
  for (int i = 0; i < half; ++i) {
    const float e = (2.0f * static_cast<float>(i)) / static_cast<float>(dim);
    const float p = powf(theta, e);
    for (int pos = 0; pos < max_pos; ++pos) {
      const float angle = static_cast<float>(pos) / p;
      float* cs = cos_sin + (static_cast<long long>(pos) * half + i) * 2;
      cs[0] = cosf(angle);
      cs[1] = sinf(angle);
    }
  }
}

}  // namespace uocr
