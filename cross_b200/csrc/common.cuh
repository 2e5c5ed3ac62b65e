// Shared device helpers for the CROSS CKKS hot path on B200 (sm_100a).
#pragma once

#include <cstdint>
#include <cstddef>
#include <cuda_runtime.h>

#include "../../include/cross_b200.h"

namespace cross {

// Per-limb Barrett constants, exactly the ones of jaxite_word
// finite_field.py:177-185: s = 2*ceil(log2 q), w = min(s, 32), s_w = s - w,
// m = floor(2^s / q).  Computed on the host (Python) and passed in.
struct ModC {
  uint64_t q;
  uint64_t m;
  uint32_t w;
  uint32_t s_w;
};

// finite_field.py:219-230: lazy Barrett reduction u64 -> u32 with a single
// conditional subtraction.  Every operation is the reference's uint64
// operation with the same wrap-around, so outputs (including values in
// [q, 2q)) are bit-identical.
__device__ __forceinline__ uint32_t barrett(uint64_t z, const ModC& c) {
  const uint64_t z1 = z & 0xFFFFFFFFull;
  const uint64_t z2 = z >> c.w;
  uint64_t t = ((z1 * c.m) >> c.w) + z2 * c.m;
  t >>= c.s_w;
  z -= t * c.q;
  return (uint32_t)(z >= c.q ? z - c.q : z);
}

// Specialisation for w == 32 and m < 2^32 (every modulus with
// 2^16 <= q < 2^31): (z1*m) >> 32 is the high word of a 32x32 product and
// z2*m a 32x32->64 product, so the result equals barrett() exactly.
__device__ __forceinline__ uint32_t barrett_w32(uint64_t z, uint32_t q, uint32_t m, uint32_t s_w) {
  const uint32_t zlo = (uint32_t)z;
  const uint32_t zhi = (uint32_t)(z >> 32);
  uint64_t t = (uint64_t)__umulhi(zlo, m) + (uint64_t)zhi * m;
  t >>= s_w;
  z -= t * (uint64_t)q;
  return (uint32_t)(z >= q ? z - q : z);
}

__device__ __forceinline__ uint32_t barrett_any(uint64_t z, const ModC& c) {
  if (c.w == 32 && c.m < (1ull << 32)) return barrett_w32(z, (uint32_t)c.q, (uint32_t)c.m, c.s_w);
  return barrett(z, c);
}

// Per-modulus constants of the Montgomery and BAT-lazy reductions, derived
// from q on the host (make_varc):
//   qinv = q^-1 mod 2^32          MontgomeryContext.moduli_inv_32 (finite_field.py:72)
//   winv = 2^-32 mod q            MontgomeryContext.w_inv         (finite_field.py:67)
//   r[i] = 2^(32 + 8 i) mod q     BATLazyContext.R rows as words  (finite_field.py:363-370)
struct VarC {
  uint32_t q;
  uint32_t qinv;
  uint32_t winv;
  uint32_t pad;
  uint32_t r[4];
};

// MontgomeryContext.modular_reduction (finite_field.py:94-154):
// t = z_lo q^-1 mod 2^32, result (z_hi + q - hi32(t q)) mod 2^32.  The
// reference assembles hi32(t q) from four 16 x 16-bit partial products; the
// 32 x 32 high word is the same integer.  Lazy: the result lies in [1, 2q)
// when z_hi < q.
__device__ __forceinline__ uint32_t montgomery(uint64_t z, uint32_t q, uint32_t qinv) {
  const uint32_t t = (uint32_t)z * qinv;
  return (uint32_t)(z >> 32) + q - __umulhi(t, q);
}

// BATLazyContext.modular_reduction (finite_field.py:384-425): with z split
// into its low word A and the bytes B_i of its high word,
// sum_j (sum_i B_i R[i][j] + A_j) << 8j = A + sum_i B_i (2^(32+8i) mod q),
// exactly (every byte lane stays below 2^32).  uint64 result, congruent to z.
__device__ __forceinline__ uint64_t bat_lazy(uint64_t z, const uint32_t* r) {
  const uint32_t hi = (uint32_t)(z >> 32);
  return (z & 0xFFFFFFFFull) + (uint64_t)(hi & 0xFFu) * r[0] + (uint64_t)((hi >> 8) & 0xFFu) * r[1] +
         (uint64_t)((hi >> 16) & 0xFFu) * r[2] + (uint64_t)(hi >> 24) * r[3];
}

// ShoupContext.modular_reduction (finite_field.py:305-330) cast to uint32:
// (z - (z_s >> 32) q) mod 2^32 depends only on the low word of z and of
// t = z_s >> 32.
__device__ __forceinline__ uint32_t shoup(uint32_t z_lo, uint32_t t, uint32_t q) { return z_lo - t * q; }

// Byte recombination of the BAT contraction (ntt_mm.py:33-37):
// sum_p acc_p << 8p in uint64.
__device__ __forceinline__ uint64_t combine4(uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3) {
  return (uint64_t)a0 + ((uint64_t)a1 << 8) + ((uint64_t)a2 << 16) + ((uint64_t)a3 << 24);
}

}  // namespace cross

// ---------------------------------------------------------------------------
// Host-side error plumbing shared by every translation unit.
// ---------------------------------------------------------------------------
namespace cross {
void set_error(const char* fmt, ...);
int fail_cuda(cudaError_t e, const char* where);
void count_launch(unsigned n = 1);
}  // namespace cross

#define CROSS_CHECK_CUDA(expr)                                        \
  do {                                                                \
    cudaError_t _e = (expr);                                          \
    if (_e != cudaSuccess) return ::cross::fail_cuda(_e, #expr);      \
  } while (0)

#define CROSS_REQUIRE(cond, ...)                                      \
  do {                                                                \
    if (!(cond)) {                                                    \
      ::cross::set_error(__VA_ARGS__);                                \
      return CROSS_ERR_INVALID_ARG;                                   \
    }                                                                 \
  } while (0)
