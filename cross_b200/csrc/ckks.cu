// CKKS client side (ckks_ctx.py, key_gen.py): the special FFTs, encode
// quantisation, encryption, decryption, CRT recombination and decode scaling.
//
// Double-precision steps reproduce CPython's evaluation exactly: every complex
// product is (a.re b.re - a.im b.im, a.re b.im + a.im b.re) and every sum is
// taken with __dmul_rn / __dadd_rn / __dsub_rn, which the compiler never
// contracts into fused multiply-adds; the twiddles are the caller's
// exp(2 pi i k / m) values.  Integer steps use the reference's modular
// formulas with results fully reduced (Python's % on non-negative values).
#include "internal.hpp"

namespace cross {

namespace {

constexpr int CK_THREADS = 256;
constexpr int CRT_MAX_WORDS = 66;   // big-integer words per coefficient (M <= 64 moduli below 2^31)

unsigned ck_blocks(int64_t n) {
  int64_t b = (n + CK_THREADS - 1) / CK_THREADS;
  if (b < 1) b = 1;
  return (unsigned)(b > (1 << 30) ? (1 << 30) : b);
}

__device__ __forceinline__ double2 cadd(double2 a, double2 b) { return make_double2(__dadd_rn(a.x, b.x), __dadd_rn(a.y, b.y)); }
__device__ __forceinline__ double2 csub(double2 a, double2 b) { return make_double2(__dsub_rn(a.x, b.x), __dsub_rn(a.y, b.y)); }
__device__ __forceinline__ double2 cmul(double2 a, double2 b) {
  return make_double2(__dsub_rn(__dmul_rn(a.x, b.x), __dmul_rn(a.y, b.y)),
                      __dadd_rn(__dmul_rn(a.x, b.y), __dmul_rn(a.y, b.x)));
}

// One radix-2 stage of FFTSpecialInv (DIF, ckks_ctx.py:62-74) or FFTSpecial
// (DIT, ckks_ctx.py:98-110) over `batch` vectors of nh values.
template <bool INV>
__global__ void k_fft_stage(double2* __restrict__ v, int64_t batch, int nh, int length, int m,
                            const double2* __restrict__ roots, const uint32_t* __restrict__ rot) {
  const int half = length >> 1, lenq = length << 2, step = m / lenq;
  const int64_t per = nh >> 1, total = batch * per;
  for (int64_t t = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; t < total; t += (int64_t)gridDim.x * blockDim.x) {
    const int64_t b = t / per;
    const int k = (int)(t - b * per);
    const int i = (k / half) * length, j = k % half;
    double2* a = v + b * nh;
    const int mod = (int)(rot[j] % (uint32_t)lenq);
    if (INV) {
      const int idx = ((lenq - mod) % lenq) * step;
      const double2 u = a[i + j], w = a[i + j + half];
      a[i + j] = cadd(u, w);
      a[i + j + half] = cmul(csub(u, w), roots[idx]);
    } else {
      const int idx = mod * step;
      const double2 u = a[i + j], w = cmul(a[i + j + half], roots[idx]);
      a[i + j] = cadd(u, w);
      a[i + j + half] = csub(u, w);
    }
  }
}

// _bitrev_inplace (ckks_ctx.py:35-45): swap i and bitrev(i) for i < bitrev(i);
// with `scale` (FFTSpecialInv's 1/nh, ckks_ctx.py:76-78) applied to both first.
__global__ void k_fft_bitrev(double2* __restrict__ v, int64_t batch, int nh, int bits, int scale_it, double scale) {
  const int64_t total = batch * nh;
  for (int64_t t = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; t < total; t += (int64_t)gridDim.x * blockDim.x) {
    const int64_t b = t / nh;
    const int i = (int)(t - b * nh);
    const int j = bits ? (int)(__brev((unsigned)i) >> (32 - bits)) : 0;
    if (i > j) continue;
    double2* a = v + b * nh;
    double2 x = a[i], y = a[j];
    if (scale_it) {
      x = make_double2(__dmul_rn(x.x, scale), __dmul_rn(x.y, scale));
      y = make_double2(__dmul_rn(y.x, scale), __dmul_rn(y.y, scale));
    }
    a[i] = y;
    a[j] = x;
  }
}

// max |scale * v| (ckks_ctx.py:357-365 takes ceil(log2) of each; the
// largest value gives the largest ceil(log2)).  Non-negative doubles order as
// their bit patterns, so an unsigned atomic max is exact.
__global__ void k_max_abs_scaled(const double* __restrict__ v, int64_t n, double scale,
                                 unsigned long long* __restrict__ out) {
  unsigned long long best = 0;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
    best = max(best, (unsigned long long)__double_as_longlong(fabs(__dmul_rn(scale, v[i]))));
  for (int o = 16; o; o >>= 1) best = max(best, __shfl_xor_sync(0xffffffffu, best, o));
  if ((threadIdx.x & 31) == 0) atomicMax(out, best);
}

// ckks_ctx.py:356-387 for coefficient i of slot_to_coeffs(y) (real parts of
// the nh slots, then their imaginary parts) and every tower:
// x = nearest_int(scale v / 2^la); fit_to_native_vector maps x to x mod q
// (x < 0 arrives as x + MAX_INT_64, which the map returns to x + q); times
// 2^la and times factor[t] mod q.  y: nh complex values; out: (M, 2 nh).
__global__ void k_ckks_quantize(const double* __restrict__ yv, int nh, double scale, double approx, int la,
                                const ModC* __restrict__ mods, int M, const uint32_t* __restrict__ factor,
                                uint32_t* __restrict__ out) {
  const int64_t n = 2 * (int64_t)nh;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    const double v = i < nh ? yv[2 * i] : yv[2 * (i - nh) + 1];
    const double y = __ddiv_rn(__dmul_rn(scale, v), approx);
    const long long x = y >= 0.0 ? (long long)floor(__dadd_rn(y, 0.5)) : -(long long)floor(__dadd_rn(-y, 0.5));
    for (int t = 0; t < M; ++t) {
      const uint64_t q = mods[t].q;
      long long r = x % (long long)q;
      uint64_t u = (uint64_t)(r < 0 ? r + (long long)q : r);
      if (la > 0) {
        uint64_t p2 = 1;   // 2^la mod q
        for (int k = 0; k < la; ++k) p2 = (p2 << 1) % q;
        u = u * p2 % q;
      }
      if (factor) u = u * factor[t] % q;
      out[(int64_t)t * n + i] = (uint32_t)u;
    }
  }
}

// gen_rns_polynomial: signed integer coefficients reduced into every tower
// (Python's %: non-negative results).  out: (M, n).
__global__ void k_rns_from_signed(const long long* __restrict__ x, int64_t n, int M, const ModC* __restrict__ mods,
                                  uint32_t* __restrict__ out) {
  const int64_t total = (int64_t)M * n;
  for (int64_t k = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; k < total; k += (int64_t)gridDim.x * blockDim.x) {
    const long long q = (long long)mods[k / n].q;
    const long long r = x[k % n] % q;
    out[k] = (uint32_t)(r < 0 ? r + q : r);
  }
}

// x[t][i] = (x[t][i] * tab[t][i]) mod q_t, fully reduced (tab == nullptr: x mod q_t).
__global__ void k_mul_reduce_lm(const uint32_t* __restrict__ x, const uint32_t* __restrict__ tab,
                                uint32_t* __restrict__ out, int64_t n, int M, const ModC* __restrict__ mods) {
  const int64_t total = (int64_t)M * n;
  for (int64_t k = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; k < total; k += (int64_t)gridDim.x * blockDim.x) {
    const uint64_t q = mods[k / n].q;
    uint64_t v = x[k];
    v = tab ? v * tab[k] % q : v % q;
    out[k] = (uint32_t)v;
  }
}

// ckks_ctx.py:264-294: res = c0 + sum_{i >= 1} c_i s^i (mod q, reduced every
// step).  c: (elements, n, M); s: (M, n); out: (M, n) limb-major.
__global__ void k_ckks_decrypt_sum(const uint32_t* __restrict__ c, int elements, const uint32_t* __restrict__ s,
                                   uint32_t* __restrict__ out, int64_t n, int M, const ModC* __restrict__ mods) {
  const int64_t total = (int64_t)M * n;
  for (int64_t k = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; k < total; k += (int64_t)gridDim.x * blockDim.x) {
    const int t = (int)(k / n);
    const int64_t d = k - (int64_t)t * n;
    const uint64_t q = mods[t].q;
    const uint64_t sv = s[k];
    uint64_t res = c[d * M + t];
    uint64_t sp = sv;
    for (int e = 1; e < elements; ++e) {
      const uint64_t term = (uint64_t)c[((int64_t)e * n + d) * M + t] * sp % q;
      res = (res + term) % q;
      if (e + 1 < elements) sp = sp * sv % q;
    }
    out[k] = (uint32_t)res;
  }
}

// ckks_ctx.py:214-228: c0 = ((v pk0 + ns e0) mod q + m) mod q, c1 = (v pk1 + ns e1) mod q.
// v, e0, e1, pk0, pk1: (M, n); m, c0, c1: (n, M).
__global__ void k_ckks_encrypt(const uint32_t* __restrict__ m, const uint32_t* __restrict__ v,
                               const uint32_t* __restrict__ e0, const uint32_t* __restrict__ e1,
                               const uint32_t* __restrict__ pk0, const uint32_t* __restrict__ pk1, uint64_t ns,
                               uint32_t* __restrict__ c0, uint32_t* __restrict__ c1, int64_t n, int M,
                               const ModC* __restrict__ mods) {
  const int64_t total = (int64_t)M * n;
  for (int64_t k = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; k < total; k += (int64_t)gridDim.x * blockDim.x) {
    const int t = (int)(k / n);
    const int64_t d = k - (int64_t)t * n;
    const uint64_t q = mods[t].q, nsq = ns % q;
    const uint64_t a = ((uint64_t)v[k] * pk0[k] % q + nsq * e0[k] % q) % q;
    c0[d * M + t] = (uint32_t)((a + m[d * M + t]) % q);
    c1[d * M + t] = (uint32_t)(((uint64_t)v[k] * pk1[k] % q + nsq * e1[k] % q) % q);
  }
}

// key_gen.py:328-337: b = ((e ns) mod q - (a s) mod q) mod q, all (M, n).
__global__ void k_pke_b(const uint32_t* __restrict__ e, const uint32_t* __restrict__ a, const uint32_t* __restrict__ s,
                        uint64_t ns, uint32_t* __restrict__ b, int64_t n, int M, const ModC* __restrict__ mods) {
  const int64_t total = (int64_t)M * n;
  for (int64_t k = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; k < total; k += (int64_t)gridDim.x * blockDim.x) {
    const uint64_t q = mods[k / n].q;
    const uint64_t x = (uint64_t)e[k] * (ns % q) % q, y = (uint64_t)a[k] * s[k] % q;
    b[k] = (uint32_t)(x >= y ? x - y : x + q - y);
  }
}

// modulus_switch (key_gen.py:77-105) of one tower's coefficients v (residues
// mod q_from) into every target modulus p_t: v below (q_from + 1) / 2 stays,
// larger v becomes v - q_from; out (M, n) holds that signed value mod p_t,
// the residue the following negacyclic transform reduces it to.
__global__ void k_mod_switch_lift(const uint32_t* __restrict__ v, int64_t n, uint32_t q_from, int M,
                                  const ModC* __restrict__ mods, uint32_t* __restrict__ out) {
  const int64_t total = (int64_t)M * n;
  const uint32_t thr = (uint32_t)(((uint64_t)q_from + 1) / 2);
  for (int64_t k = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; k < total; k += (int64_t)gridDim.x * blockDim.x) {
    const long long p = (long long)mods[k / n].q;
    const uint32_t x = v[k % n];
    long long c = x < thr ? (long long)x : (long long)x - (long long)q_from;
    c %= p;
    out[k] = (uint32_t)(c < 0 ? c + p : c);
  }
}

// key_switch_gen's b (key_gen.py:228-246) for one part: rows i of Q + P,
// b = (-a s mod q + [P s_old mod q for start <= i < end] + ns e mod q) mod q.
// a, e, s, b: (Q + P, n); s_old: (Q, n); p_mod_q: (Q).
__global__ void k_ks_key_b(const uint32_t* __restrict__ a, const uint32_t* __restrict__ e,
                           const uint32_t* __restrict__ s, const uint32_t* __restrict__ s_old,
                           const uint32_t* __restrict__ p_mod_q, int start, int end, uint64_t ns,
                           uint32_t* __restrict__ b, int64_t n, int M, const ModC* __restrict__ mods) {
  const int64_t total = (int64_t)M * n;
  for (int64_t k = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; k < total; k += (int64_t)gridDim.x * blockDim.x) {
    const int i = (int)(k / n);
    const uint64_t q = mods[i].q;
    const uint64_t as = (uint64_t)a[k] * s[k] % q;
    uint64_t r = (as ? q - as : 0) + (uint64_t)e[k] * (ns % q) % q;
    if (i >= start && i < end) r += (uint64_t)p_mod_q[i] * s_old[k] % q;
    b[k] = (uint32_t)(r % q);
  }
}

// ---------------------------------------------------------------------------
// Big integers: little-endian uint32 words.
// ---------------------------------------------------------------------------
__device__ __forceinline__ int cmp_words(const uint32_t* a, const uint32_t* b, int W) {
  for (int k = W - 1; k >= 0; --k)
    if (a[k] != b[k]) return a[k] < b[k] ? -1 : 1;
  return 0;
}
__device__ __forceinline__ void sub_words(uint32_t* a, const uint32_t* b, int W) {   // a -= b (a >= b)
  uint64_t borrow = 0;
  for (int k = 0; k < W; ++k) {
    const uint64_t d = (uint64_t)a[k] - b[k] - borrow;
    a[k] = (uint32_t)d;
    borrow = (d >> 63) & 1;
  }
}

// _crt_combine_rns_plaintext (ckks_ctx.py:517-545) for one coefficient:
// X = sum_i ((r_i mod q_i) (Q/q_i)^-1 mod q_i)(Q/q_i) mod Q.  The sum is
// formed exactly; floor(X / Q) is estimated from sum_i v_i / q_i (error far
// below 1), one less than the estimate is subtracted as a multiple of Q, and
// at most three conditional subtractions finish the reduction.  The
// reference's X % Q of sum_i (r_i mod q_i) (Q/q_i) inv_i equals this value.
__device__ void crt_one(const uint32_t* __restrict__ r, int M, const ModC* __restrict__ mods,
                        const uint32_t* __restrict__ inv, const uint32_t* __restrict__ mi, const uint32_t* __restrict__ Q,
                        int W, uint32_t* acc) {
  for (int k = 0; k <= W; ++k) acc[k] = 0;
  double est = 0.0;
  for (int i = 0; i < M; ++i) {
    const uint64_t q = mods[i].q;
    const uint64_t vi = (uint64_t)(r[i] % q) * inv[i] % q;
    est += (double)vi / (double)q;
    uint64_t carry = 0;
    const uint32_t* w = mi + (int64_t)i * W;
    for (int k = 0; k < W; ++k) {
      const uint64_t p = (uint64_t)w[k] * vi + acc[k] + carry;
      acc[k] = (uint32_t)p;
      carry = p >> 32;
    }
    acc[W] += (uint32_t)carry;
  }
  // subtract (floor(est) - 1) Q when positive
  const long long k0 = (long long)floor(est) - 1;
  if (k0 > 0) {
    uint64_t borrow = 0, carry = 0;
    for (int k = 0; k <= W; ++k) {
      const uint64_t p = (k < W ? (uint64_t)Q[k] * (uint64_t)k0 : 0) + carry;
      carry = p >> 32;
      const uint64_t d = (uint64_t)acc[k] - (uint32_t)p - borrow;
      acc[k] = (uint32_t)d;
      borrow = (d >> 63) & 1;
    }
  }
  for (int it = 0; it < 3; ++it) {
    if (acc[W] == 0 && cmp_words(acc, Q, W) < 0) break;
    uint64_t borrow = 0;
    for (int k = 0; k <= W; ++k) {
      const uint64_t d = (uint64_t)acc[k] - (k < W ? Q[k] : 0u) - borrow;
      acc[k] = (uint32_t)d;
      borrow = (d >> 63) & 1;
    }
  }
}

__global__ void k_crt_combine(const uint32_t* __restrict__ rns, int64_t n, int M, const ModC* __restrict__ mods,
                              const uint32_t* __restrict__ inv, const uint32_t* __restrict__ mi,
                              const uint32_t* __restrict__ Q, int W, uint32_t* __restrict__ out) {
  uint32_t acc[CRT_MAX_WORDS + 1];
  for (int64_t d = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; d < n; d += (int64_t)gridDim.x * blockDim.x) {
    crt_one(rns + d * M, M, mods, inv, mi, Q, W, acc);
    for (int k = 0; k < W; ++k) out[d * W + k] = acc[k];
  }
}

// float(X) for a non-negative big integer, rounded to nearest-even (CPython's
// int.__float__): the top 64 bits with the lower bits folded into a sticky
// bit, converted by the hardware's round-to-nearest, then scaled by a power
// of two (exact).  Sets *overflow when X >= 2^1024 (CPython raises).
__device__ double words_to_double(const uint32_t* x, int W, int* overflow) {
  int t = W - 1;
  while (t >= 0 && x[t] == 0) --t;
  if (t < 0) return 0.0;
  const int msb = 32 * t + 31 - __clz(x[t]);
  if (msb < 64) {
    const uint64_t lo = x[0] | (W > 1 ? (uint64_t)x[1] << 32 : 0ull);
    return __ull2double_rn(lo);
  }
  if (msb >= 1024) {
    *overflow = 1;
    return 0.0;
  }
  const int lo = msb - 63, w0 = lo >> 5, sh = lo & 31;
  const uint64_t a = x[w0], b = w0 + 1 < W ? x[w0 + 1] : 0u, c = w0 + 2 < W ? x[w0 + 2] : 0u;
  uint64_t hi = sh ? (a >> sh) | (b << (32 - sh)) | (c << (64 - sh)) : a | (b << 32);
  bool sticky = sh && (a & ((1u << sh) - 1u));
  for (int k = 0; k < w0 && !sticky; ++k) sticky = x[k] != 0;
  return ldexp(__ull2double_rn(hi | (sticky ? 1ull : 0ull)), lo);
}

// ckks_ctx.py:421-441 for slot i: the value of coefficient i (real part) and
// i + nh (imaginary part): centred at Q/2, times sf_pre, truncated toward 0.
__global__ void k_decode_scale(const uint32_t* __restrict__ x, int W, const uint32_t* __restrict__ Q,
                               const uint32_t* __restrict__ half, double sf_pre, int slots, int nh,
                               double2* __restrict__ out, int* __restrict__ overflow) {
  uint32_t tmp[CRT_MAX_WORDS];
  for (int64_t k = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; k < 2 * (int64_t)slots;
       k += (int64_t)gridDim.x * blockDim.x) {
    const int i = (int)(k >> 1), part = (int)(k & 1);
    const uint32_t* v = x + (int64_t)(i + part * nh) * W;
    const bool neg = cmp_words(v, half, W) > 0;
    for (int w = 0; w < W; ++w) tmp[w] = neg ? Q[w] : v[w];
    if (neg) sub_words(tmp, v, W);
    double r = __dmul_rn(words_to_double(tmp, W, overflow), sf_pre);
    if (neg) r = -r;
    r = trunc(r);
    double* o = reinterpret_cast<double*>(out + i);
    o[part] = r;
  }
}

// Sum of one double per thread over a block of SD_THREADS threads (warp
// shuffles, then the warp totals); every thread receives the total.
constexpr int SD_THREADS = 1024;
__device__ double block_sum(double v, double* red) {
  for (int o = 16; o; o >>= 1) v = __dadd_rn(v, __shfl_down_sync(0xffffffffu, v, o));
  __syncthreads();
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
  __syncthreads();
  if (threadIdx.x < 32) {
    double w = red[threadIdx.x];
    for (int o = 16; o; o >>= 1) w = __dadd_rn(w, __shfl_down_sync(0xffffffffu, w, o));
    if (threadIdx.x == 0) red[0] = w;
  }
  __syncthreads();
  return red[0];
}

// ckks_ctx.py:458-481 (_stddev): the mean and variance of cur - conj(cur)
// over slots 0 .. s/2, as one block with parallel sums.  CPython's sum()
// compensates its own float additions, so no summation order reproduces the
// reference's last bits; the estimate only decides whether decode raises.
// cur: the slot values; out: the standard deviation estimate.
__global__ void __launch_bounds__(SD_THREADS) k_decode_stddev(const double2* __restrict__ cur, int s,
                                                              double* __restrict__ out) {
  __shared__ double red[SD_THREADS / 32];
  if (s == 1) {
    if (threadIdx.x == 0) *out = cur[0].y;
    return;
  }
  auto cv = [&](int i) -> double2 {
    const double2 c = i == 0 ? make_double2(cur[0].x, -cur[0].y) : make_double2(-cur[s - i].y, -cur[s - i].x);
    return csub(cur[i], c);
  };
  const double dslots = 2.0 * s;
  double part = 0.0;
  for (int i = 1 + threadIdx.x; i < s / 2; i += SD_THREADS) {
    const double2 c = cv(i);
    part = __dadd_rn(part, __dadd_rn(c.x, c.y));
  }
  double mean = __dmul_rn(2.0, block_sum(part, red));
  mean = __dadd_rn(mean, cv(0).y);
  mean = __dadd_rn(mean, __dmul_rn(2.0, cv(s / 2).x));
  mean = __ddiv_rn(mean, __dsub_rn(dslots, 1.0));
  part = 0.0;
  for (int i = 1 + threadIdx.x; i < s / 2; i += SD_THREADS) {
    const double2 c = cv(i);
    const double a = __dsub_rn(c.x, mean), b = __dsub_rn(c.y, mean);
    part = __dadd_rn(part, __dadd_rn(__dmul_rn(a, a), __dmul_rn(b, b)));
  }
  double var = __dmul_rn(2.0, block_sum(part, red));
  if (threadIdx.x == 0) {
    const double a0 = __dsub_rn(cv(0).y, mean), a1 = __dsub_rn(cv(s / 2).x, mean);
    var = __dadd_rn(var, __dmul_rn(a0, a0));
    var = __dadd_rn(var, __dmul_rn(2.0, __dmul_rn(a1, a1)));
    var = __ddiv_rn(var, __dsub_rn(dslots, 2.0));
    *out = __dmul_rn(0.5, __dsqrt_rn(var));
  }
}

// ckks_ctx.py:496-505: cur[i] = (re_i s + conj_i.re s, im_i s + conj_i.im s).
__global__ void k_decode_combine(const double2* __restrict__ in, double2* __restrict__ out, int s, double scale) {
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < s; i += gridDim.x * blockDim.x) {
    const double2 z = in[i];
    double2 c;
    if (i == 0) {
      c = make_double2(z.x, -z.y);
    } else {
      const double2 w = in[s - i];
      c = make_double2(-w.y, -w.x);
    }
    out[i] = make_double2(__dadd_rn(__dmul_rn(z.x, scale), __dmul_rn(c.x, scale)),
                          __dadd_rn(__dmul_rn(z.y, scale), __dmul_rn(c.y, scale)));
  }
}

}  // namespace

}  // namespace cross

using namespace cross;

extern "C" {

int cross_fft_special(double* vals, int64_t batch, int nh, int m, const double* roots, const uint32_t* rot,
                      int inverse, double inv_scale, void* stream) {
  CROSS_REQUIRE(batch >= 0 && nh >= 1 && (nh & (nh - 1)) == 0 && m >= 4 * nh && (m & (m - 1)) == 0 &&
                    (batch == 0 || (vals && roots && rot)),
                "cross_fft_special: nh and m must be powers of two with m >= 4 nh");
  if (batch == 0) return CROSS_OK;
  cudaStream_t st = (cudaStream_t)stream;
  double2* v = reinterpret_cast<double2*>(vals);
  const double2* rt = reinterpret_cast<const double2*>(roots);
  int bits = 0;
  while ((1 << bits) < nh) ++bits;
  const unsigned g = ck_blocks(batch * (nh / 2 > 0 ? nh / 2 : 1));
  if (inverse) {
    for (int length = nh; length >= 2; length >>= 1) {
      k_fft_stage<true><<<g, CK_THREADS, 0, st>>>(v, batch, nh, length, m, rt, rot);
      count_launch();
    }
    k_fft_bitrev<<<ck_blocks(batch * nh), CK_THREADS, 0, st>>>(v, batch, nh, bits, 1, inv_scale);
    count_launch();
  } else {
    k_fft_bitrev<<<ck_blocks(batch * nh), CK_THREADS, 0, st>>>(v, batch, nh, bits, 0, 1.0);
    count_launch();
    for (int length = 2; length <= nh; length <<= 1) {
      k_fft_stage<false><<<g, CK_THREADS, 0, st>>>(v, batch, nh, length, m, rt, rot);
      count_launch();
    }
  }
  CROSS_CHECK_CUDA(cudaGetLastError());
  return CROSS_OK;
}

int cross_ckks_max_abs_scaled(const double* v, int64_t n, double scale, double* out, void* stream) {
  CROSS_REQUIRE(n >= 0 && out && (n == 0 || v), "cross_ckks_max_abs_scaled: bad argument");
  cudaStream_t st = (cudaStream_t)stream;
  CROSS_CHECK_CUDA(cudaMemsetAsync(out, 0, sizeof(double), st));
  if (n == 0) return CROSS_OK;
  const int64_t b = (n + CK_THREADS - 1) / CK_THREADS;
  k_max_abs_scaled<<<(unsigned)(b < 1024 ? b : 1024), CK_THREADS, 0, st>>>(v, n, scale, (unsigned long long*)out);
  count_launch();
  CROSS_CHECK_CUDA(cudaGetLastError());
  return CROSS_OK;
}

int cross_ckks_quantize(cross_moduli moduli, const double* y, int nh, double scale, int log_approx,
                        const uint32_t* factor, uint32_t* out, void* stream) {
  CROSS_REQUIRE(moduli && nh >= 0 && log_approx >= 0 && log_approx < 1024 && (nh == 0 || (y && out)),
                "cross_ckks_quantize: bad argument");
  if (nh == 0) return CROSS_OK;
  const double approx = ldexp(1.0, log_approx);
  k_ckks_quantize<<<ck_blocks(2 * (int64_t)nh), CK_THREADS, 0, (cudaStream_t)stream>>>(
      y, nh, scale, approx, log_approx, moduli->dev, moduli->n, factor, out);
  count_launch();
  CROSS_CHECK_CUDA(cudaGetLastError());
  return CROSS_OK;
}

int cross_mul_reduce_lm(cross_moduli moduli, const uint32_t* x, const uint32_t* tab, uint32_t* out, int64_t n,
                        void* stream) {
  CROSS_REQUIRE(moduli && n >= 0 && (n == 0 || (x && out)), "cross_mul_reduce_lm: bad argument");
  if (n == 0) return CROSS_OK;
  k_mul_reduce_lm<<<ck_blocks(n * moduli->n), CK_THREADS, 0, (cudaStream_t)stream>>>(x, tab, out, n, moduli->n,
                                                                                     moduli->dev);
  count_launch();
  CROSS_CHECK_CUDA(cudaGetLastError());
  return CROSS_OK;
}

int cross_rns_from_signed(cross_moduli moduli, const int64_t* x, int64_t n, uint32_t* out, void* stream) {
  CROSS_REQUIRE(moduli && n >= 0 && (n == 0 || (x && out)), "cross_rns_from_signed: bad argument");
  if (n == 0) return CROSS_OK;
  k_rns_from_signed<<<ck_blocks(n * moduli->n), CK_THREADS, 0, (cudaStream_t)stream>>>(
      reinterpret_cast<const long long*>(x), n, moduli->n, moduli->dev, out);
  count_launch();
  CROSS_CHECK_CUDA(cudaGetLastError());
  return CROSS_OK;
}

int cross_mod_switch_lift(const uint32_t* v, int64_t n, uint32_t q_from, cross_moduli to, uint32_t* out,
                          void* stream) {
  CROSS_REQUIRE(to && n >= 0 && q_from > 1 && (n == 0 || (v && out)), "cross_mod_switch_lift: bad argument");
  if (n == 0) return CROSS_OK;
  k_mod_switch_lift<<<ck_blocks(n * to->n), CK_THREADS, 0, (cudaStream_t)stream>>>(v, n, q_from, to->n, to->dev, out);
  count_launch();
  CROSS_CHECK_CUDA(cudaGetLastError());
  return CROSS_OK;
}

int cross_ks_key_b(cross_moduli moduli, const uint32_t* a, const uint32_t* e, const uint32_t* s, const uint32_t* s_old,
                   const uint32_t* p_mod_q, int start, int end, uint64_t noise_scale, uint32_t* b, int64_t n,
                   void* stream) {
  CROSS_REQUIRE(moduli && n >= 0 && start >= 0 && end >= start && end <= moduli->n &&
                    (n == 0 || (a && e && s && b && (start == end || (s_old && p_mod_q)))),
                "cross_ks_key_b: bad argument");
  if (n == 0) return CROSS_OK;
  k_ks_key_b<<<ck_blocks(n * moduli->n), CK_THREADS, 0, (cudaStream_t)stream>>>(a, e, s, s_old, p_mod_q, start, end,
                                                                                noise_scale, b, n, moduli->n,
                                                                                moduli->dev);
  count_launch();
  CROSS_CHECK_CUDA(cudaGetLastError());
  return CROSS_OK;
}

int cross_ckks_decrypt_sum(cross_moduli moduli, const uint32_t* c, int elements, const uint32_t* s, uint32_t* out,
                           int64_t n, void* stream) {
  CROSS_REQUIRE(moduli && elements >= 1 && n >= 0 && (n == 0 || (c && s && out)), "cross_ckks_decrypt_sum: bad argument");
  if (n == 0) return CROSS_OK;
  k_ckks_decrypt_sum<<<ck_blocks(n * moduli->n), CK_THREADS, 0, (cudaStream_t)stream>>>(c, elements, s, out, n,
                                                                                        moduli->n, moduli->dev);
  count_launch();
  CROSS_CHECK_CUDA(cudaGetLastError());
  return CROSS_OK;
}

int cross_ckks_encrypt(cross_moduli moduli, const uint32_t* m, const uint32_t* v, const uint32_t* e0,
                       const uint32_t* e1, const uint32_t* pk0, const uint32_t* pk1, uint64_t noise_scale,
                       uint32_t* c0, uint32_t* c1, int64_t n, void* stream) {
  CROSS_REQUIRE(moduli && n >= 0 && (n == 0 || (m && v && e0 && e1 && pk0 && pk1 && c0 && c1)),
                "cross_ckks_encrypt: bad argument");
  if (n == 0) return CROSS_OK;
  k_ckks_encrypt<<<ck_blocks(n * moduli->n), CK_THREADS, 0, (cudaStream_t)stream>>>(m, v, e0, e1, pk0, pk1, noise_scale,
                                                                                    c0, c1, n, moduli->n, moduli->dev);
  count_launch();
  CROSS_CHECK_CUDA(cudaGetLastError());
  return CROSS_OK;
}

int cross_pke_b(cross_moduli moduli, const uint32_t* e, const uint32_t* a, const uint32_t* s, uint64_t noise_scale,
                uint32_t* b, int64_t n, void* stream) {
  CROSS_REQUIRE(moduli && n >= 0 && (n == 0 || (e && a && s && b)), "cross_pke_b: bad argument");
  if (n == 0) return CROSS_OK;
  k_pke_b<<<ck_blocks(n * moduli->n), CK_THREADS, 0, (cudaStream_t)stream>>>(e, a, s, noise_scale, b, n, moduli->n,
                                                                             moduli->dev);
  count_launch();
  CROSS_CHECK_CUDA(cudaGetLastError());
  return CROSS_OK;
}

int cross_crt_combine(cross_moduli moduli, const uint32_t* rns, int64_t n, const uint32_t* inv, const uint32_t* mi,
                      const uint32_t* q_words, int words, uint32_t* out, void* stream) {
  CROSS_REQUIRE(moduli && n >= 0 && words >= 1 && words <= CRT_MAX_WORDS && moduli->n <= 64 &&
                    (n == 0 || (rns && inv && mi && q_words && out)),
                "cross_crt_combine: bad argument (at most %d words, 64 moduli)", CRT_MAX_WORDS);
  if (n == 0) return CROSS_OK;
  k_crt_combine<<<ck_blocks(n), 128, 0, (cudaStream_t)stream>>>(rns, n, moduli->n, moduli->dev, inv, mi, q_words,
                                                               words, out);
  count_launch();
  CROSS_CHECK_CUDA(cudaGetLastError());
  return CROSS_OK;
}

int cross_ckks_decode_scale(const uint32_t* x, int words, const uint32_t* q_words, const uint32_t* half_words,
                            double sf_pre, int slots, int nh, double* out, int* overflow, void* stream) {
  CROSS_REQUIRE(words >= 1 && words <= CRT_MAX_WORDS && slots >= 0 && slots <= nh &&
                    (slots == 0 || (x && q_words && half_words && out && overflow)),
                "cross_ckks_decode_scale: bad argument");
  if (slots == 0) return CROSS_OK;
  k_decode_scale<<<ck_blocks(2 * (int64_t)slots), 128, 0, (cudaStream_t)stream>>>(
      x, words, q_words, half_words, sf_pre, slots, nh, reinterpret_cast<double2*>(out), overflow);
  count_launch();
  CROSS_CHECK_CUDA(cudaGetLastError());
  return CROSS_OK;
}

int cross_ckks_decode_stddev(const double* cur, int slots, double* out, void* stream) {
  CROSS_REQUIRE(slots >= 1 && cur && out, "cross_ckks_decode_stddev: bad argument");
  k_decode_stddev<<<1, SD_THREADS, 0, (cudaStream_t)stream>>>(reinterpret_cast<const double2*>(cur), slots, out);
  count_launch();
  CROSS_CHECK_CUDA(cudaGetLastError());
  return CROSS_OK;
}

int cross_ckks_decode_combine(const double* in, double* out, int slots, double scale, void* stream) {
  CROSS_REQUIRE(slots >= 0 && (slots == 0 || (in && out && in != out)), "cross_ckks_decode_combine: bad argument");
  if (slots == 0) return CROSS_OK;
  k_decode_combine<<<ck_blocks(slots), CK_THREADS, 0, (cudaStream_t)stream>>>(
      reinterpret_cast<const double2*>(in), reinterpret_cast<double2*>(out), slots, scale);
  count_launch();
  CROSS_CHECK_CUDA(cudaGetLastError());
  return CROSS_OK;
}

}  // extern "C"
