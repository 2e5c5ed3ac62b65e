// Elementwise modular kernels: Barrett reduction, modmul with broadcast
// tables, the HE tensor product, modular add, the Galois permutation and the
// layout conversions.  All are HBM-bound; indices are 64-bit.
#include "internal.hpp"
#include "tc_ptx.cuh"

namespace cross {

namespace {

constexpr int EW_THREADS = 256;

unsigned ew_blocks(int64_t n, int per_thread = 1) {
  int64_t b = (n + (int64_t)EW_THREADS * per_thread - 1) / ((int64_t)EW_THREADS * per_thread);
  if (b < 1) b = 1;
  return (unsigned)(b > (1 << 30) ? (1 << 30) : b);
}

template <bool U64IN>
__global__ void k_mod_reduce(const void* __restrict__ in, uint32_t* __restrict__ out, int64_t total,
                             int M, const ModC* __restrict__ mods) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    const uint64_t z = U64IN ? ((const uint64_t*)in)[i] : (uint64_t)((const uint32_t*)in)[i];
    out[i] = barrett_any(z, mods[i % M]);
  }
}

// The other finite_field.py reductions, elementwise with moduli on the last
// axis: Montgomery and Shoup to uint32, BAT-lazy to uint64.
template <int RED>
__global__ void k_mod_reduce_var(const uint64_t* __restrict__ z, const uint64_t* __restrict__ zs,
                                 void* __restrict__ out, int64_t total, int M, const VarC* __restrict__ v) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    const VarC& c = v[i % M];
    if (RED == CROSS_REDUCTION_MONTGOMERY)
      static_cast<uint32_t*>(out)[i] = montgomery(z[i], c.q, c.qinv);
    else if (RED == CROSS_REDUCTION_SHOUP)
      static_cast<uint32_t*>(out)[i] = shoup((uint32_t)z[i], (uint32_t)(zs[i] >> 32), c.q);
    else
      static_cast<uint64_t*>(out)[i] = bat_lazy(z[i], c.r);
  }
}

__global__ void k_modmul_ref(const void* __restrict__ a, int a64, const void* __restrict__ b, int b64,
                             int64_t b_rows, uint32_t* __restrict__ out, int64_t total, int M,
                             const ModC* __restrict__ mods) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int m = (int)(i % M);
    const int64_t row = i / M;
    const int64_t bi = (row % b_rows) * M + m;
    const uint64_t x = a64 ? ((const uint64_t*)a)[i] : (uint64_t)((const uint32_t*)a)[i];
    const uint64_t y = b64 ? ((const uint64_t*)b)[bi] : (uint64_t)((const uint32_t*)b)[bi];
    out[i] = barrett_any(x * y, mods[m]);
  }
}

// ciphertext.py:309-324 on (batch, 4, n, M): elements a0, a1, b0, b1.
__global__ void k_tensor_ref(const uint32_t* __restrict__ ct, uint32_t* __restrict__ o01,
                             uint32_t* __restrict__ o2, int64_t batch, int64_t per, int M,
                             const ModC* __restrict__ mods) {
  const int64_t total = batch * per;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t b = i / per, t = i % per;
    const ModC mc = mods[t % M];
    const uint32_t* base = ct + b * 4 * per + t;
    const uint64_t a0 = base[0], a1 = base[per], b0 = base[2 * per], b1 = base[3 * per];
    o01[b * 2 * per + t] = barrett_any(a0 * b0, mc);
    o01[b * 2 * per + per + t] = barrett_any(a0 * b1 + a1 * b0, mc);
    o2[b * per + t] = barrett_any(a1 * b1, mc);
  }
}

// add.py:7-27 on (E, M, n): result = a + b; result > q ? result - q : result.
__global__ void k_add_mod(const uint32_t* __restrict__ a, const uint32_t* __restrict__ b,
                          uint32_t* __restrict__ out, int64_t total, int64_t n, int M,
                          const ModC* __restrict__ mods) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    const uint32_t q = (uint32_t)mods[(i / n) % M].q;
    const uint32_t s = a[i] + b[i];
    out[i] = s > q ? s - q : s;
  }
}

// herot.py:300 jnp.take(x, coef_map, axis=2) on (polys, n, M): row gather.
__global__ void k_gather_rows(const uint32_t* __restrict__ in, const int32_t* __restrict__ map,
                              uint32_t* __restrict__ out, int64_t polys, int64_t n, int M) {
  const int64_t total = polys * n * M;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int m = (int)(i % M);
    const int64_t row = i / M;
    const int64_t p = row / n, j = row % n;
    int64_t src = map[j];
    // jnp.take's default mode: negative indices count from the end and any
    // index still outside [0, n) yields the fill value (UINT32_MAX).
    if (src < 0) src += n;
    out[i] = (src < 0 || src >= n) ? 0xFFFFFFFFu : in[(p * n + src) * M + m];
  }
}

// 32-bit index forms of the four kernels above, for launches of fewer than
// 2^31 elements (every call of the HE parameter sets): the limb of element i
// is one 32-bit remainder, and the other index splits are a 32-bit remainder
// or, for a power-of-two ring dimension (log2n >= 0), a shift and a mask,
// instead of 64-bit divisions per element.
template <bool U64IN>
__global__ void k_mod_reduce32(const void* __restrict__ in, uint32_t* __restrict__ out, uint32_t total,
                               uint32_t M, const ModC* __restrict__ mods) {
  for (uint32_t i = blockIdx.x * blockDim.x + threadIdx.x; i < total; i += gridDim.x * blockDim.x) {
    const uint64_t z = U64IN ? ((const uint64_t*)in)[i] : (uint64_t)((const uint32_t*)in)[i];
    out[i] = barrett_any(z, mods[i % M]);
  }
}

// modmul with the broadcast table: b's element for i is (i / M % b_rows) M +
// i % M = i % (b_rows M); bm = b_rows M, or 0 when b covers every row.
template <bool A64, bool B64>
__global__ void k_modmul32(const void* __restrict__ a, const void* __restrict__ b, uint32_t bm,
                           uint32_t* __restrict__ out, uint32_t total, uint32_t M, const ModC* __restrict__ mods) {
  for (uint32_t i = blockIdx.x * blockDim.x + threadIdx.x; i < total; i += gridDim.x * blockDim.x) {
    const uint32_t bi = bm ? i % bm : i;
    const uint64_t x = A64 ? ((const uint64_t*)a)[i] : (uint64_t)((const uint32_t*)a)[i];
    const uint64_t y = B64 ? ((const uint64_t*)b)[bi] : (uint64_t)((const uint32_t*)b)[bi];
    out[i] = barrett_any(x * y, mods[i % M]);
  }
}

__global__ void k_add_mod32(const uint32_t* __restrict__ a, const uint32_t* __restrict__ b,
                            uint32_t* __restrict__ out, uint32_t total, uint32_t n, int log2n, uint32_t M,
                            const ModC* __restrict__ mods) {
  for (uint32_t i = blockIdx.x * blockDim.x + threadIdx.x; i < total; i += gridDim.x * blockDim.x) {
    const uint32_t row = log2n >= 0 ? i >> log2n : i / n;
    const uint32_t q = (uint32_t)mods[row % M].q;
    const uint32_t s = a[i] + b[i];
    out[i] = s > q ? s - q : s;
  }
}

__global__ void k_gather_rows32(const uint32_t* __restrict__ in, const int32_t* __restrict__ map,
                                uint32_t* __restrict__ out, uint32_t total, uint32_t n, int log2n, uint32_t M) {
  for (uint32_t i = blockIdx.x * blockDim.x + threadIdx.x; i < total; i += gridDim.x * blockDim.x) {
    const uint32_t row = i / M, m = i - row * M;
    const uint32_t p = log2n >= 0 ? row >> log2n : row / n;
    const uint32_t j = row - p * n;
    int64_t src = map[j];
    // jnp.take's default mode, as in k_gather_rows
    if (src < 0) src += n;
    out[i] = (src < 0 || src >= (int64_t)n) ? 0xFFFFFFFFu : in[((int64_t)p * n + src) * M + m];
  }
}

// Barrett of x * y for modulus c = {q, m, s_w, forms} (cross_moduli_s::dev_f):
// the exact 32-bit remainder form when the modulus allows it and the product
// is a word below 2^31 times a residue (tc::reduce_fast2's exactness bound),
// barrett_w32 for other inputs of a w = 32 modulus, the generic form else.
// Every branch returns finite_field.py's value.
__device__ __forceinline__ uint32_t mulmod_packed(uint32_t x, uint32_t y, const uint4& c, const ModC& mc) {
  if ((c.w & 2u) && x < 0x80000000u && y < c.x) return tc::reduce_fast2(x * y, __umulhi(x, y), c.x, c.y, c.z);
  if (c.w & 1u) return barrett_w32((uint64_t)x * y, c.x, c.y, c.z);
  return barrett((uint64_t)x * y, mc);
}

// 16-byte forms of the uint32 modmul and add: four consecutive elements per
// thread, one remainder per four (their limbs follow in turn for modmul; they
// share one limb for add, whose ring dimension is a multiple of 4).  The
// launcher picks them for 16-byte aligned buffers whose sizes are multiples
// of 4 (the table period bm too).  modmul reads each limb's constants as one
// packed 16-byte record.
template <bool BCAST>
__global__ void k_modmul32v(const uint32_t* __restrict__ a, const uint32_t* __restrict__ b, uint32_t bm,
                            uint32_t* __restrict__ out, uint32_t total4, uint32_t M, const ModC* __restrict__ mods,
                            const uint4* __restrict__ fc) {
  for (uint32_t v = blockIdx.x * blockDim.x + threadIdx.x; v < total4; v += gridDim.x * blockDim.x) {
    const uint32_t i = 4 * v;
    const uint4 x = reinterpret_cast<const uint4*>(a)[v];
    const uint4 y = *reinterpret_cast<const uint4*>(b + (BCAST ? i % bm : i));
    uint32_t m = i % M;
    uint4 r;
    r.x = mulmod_packed(x.x, y.x, __ldg(fc + m), mods[m]);
    m = m + 1 == M ? 0 : m + 1;
    r.y = mulmod_packed(x.y, y.y, __ldg(fc + m), mods[m]);
    m = m + 1 == M ? 0 : m + 1;
    r.z = mulmod_packed(x.z, y.z, __ldg(fc + m), mods[m]);
    m = m + 1 == M ? 0 : m + 1;
    r.w = mulmod_packed(x.w, y.w, __ldg(fc + m), mods[m]);
    reinterpret_cast<uint4*>(out)[v] = r;
  }
}

__global__ void k_add_mod32v(const uint32_t* __restrict__ a, const uint32_t* __restrict__ b,
                             uint32_t* __restrict__ out, uint32_t total4, uint32_t n, int log2n, uint32_t M,
                             const ModC* __restrict__ mods) {
  for (uint32_t v = blockIdx.x * blockDim.x + threadIdx.x; v < total4; v += gridDim.x * blockDim.x) {
    const uint32_t i = 4 * v;
    const uint32_t row = log2n >= 0 ? i >> log2n : i / n;
    const uint32_t q = (uint32_t)mods[row % M].q;
    const uint4 x = reinterpret_cast<const uint4*>(a)[v], y = reinterpret_cast<const uint4*>(b)[v];
    uint4 s = make_uint4(x.x + y.x, x.y + y.y, x.z + y.z, x.w + y.w);
    s.x = s.x > q ? s.x - q : s.x;
    s.y = s.y > q ? s.y - q : s.y;
    s.z = s.z > q ? s.z - q : s.z;
    s.w = s.w > q ? s.w - q : s.w;
    reinterpret_cast<uint4*>(out)[v] = s;
  }
}

bool aligned16(const void* p) { return ((uintptr_t)p & 15) == 0; }

int log2_or_neg(int64_t n) { return n > 0 && (n & (n - 1)) == 0 ? __builtin_ctzll((unsigned long long)n) : -1; }
constexpr int64_t EW32_LIMIT = (int64_t)1 << 31;

// Batched transpose (batch, rows, cols) -> (batch, cols, rows) through a
// 32x33 shared tile (coalesced on both sides).
__global__ void k_transpose(const uint32_t* __restrict__ in, uint32_t* __restrict__ out, int64_t rows,
                            int64_t cols) {
  __shared__ uint32_t tile[32][33];
  const int64_t b = blockIdx.z;
  const int64_t r0 = (int64_t)blockIdx.y * 32, c0 = (int64_t)blockIdx.x * 32;
  const uint32_t* src = in + b * rows * cols;
  uint32_t* dst = out + b * rows * cols;
  for (int i = threadIdx.y; i < 32; i += blockDim.y) {
    const int64_t r = r0 + i, c = c0 + threadIdx.x;
    if (r < rows && c < cols) tile[i][threadIdx.x] = src[r * cols + c];
  }
  __syncthreads();
  for (int i = threadIdx.y; i < 32; i += blockDim.y) {
    const int64_t c = c0 + i, r = r0 + threadIdx.x;
    if (r < rows && c < cols) dst[c * rows + r] = tile[threadIdx.x][i];
  }
}

// Transpose between the reference layout (P, N, L) (limbs innermost) and the
// limb-major layout (P, L, N) for a small limb count L.  A block moves TT
// consecutive positions of one polynomial: TT * L contiguous words on the
// reference side, L runs of TT contiguous words on the limb-major side; both
// sides are read and written fully coalesced through a padded shared tile
// [TT][L + 1].  (t, l) = divmod(k, L) uses a float reciprocal: k < TT * L <=
// 2^13 and the fractional part of (k + 0.5) / L is at least 0.5 / L, so the
// floor is exact.
constexpr int TT = 128;
constexpr int TT_MAX_L = 64;
template <bool TO_LM>
__global__ void __launch_bounds__(256) k_transpose_ref(const uint32_t* __restrict__ in, uint32_t* __restrict__ out,
                                                      int64_t n, int L, int64_t tiles) {
  extern __shared__ uint4 sm4[];
  uint32_t* sm = reinterpret_cast<uint32_t*>(sm4);
  // Row pitch of the tile: odd, so the limb-major side (consecutive t, fixed l)
  // is free of bank conflicts.  For odd L the pitch is L itself and the tile
  // is the contiguous reference-layout run, read and written as 16-byte words.
  const int ld = (L & 1) ? L : L + 1;
  const bool flat = ld == L;
  const int per = TT * L;
  const float inv = 1.0f / (float)L;
  const int64_t tiles_per_poly = n / TT;
  for (int64_t tile = blockIdx.x; tile < tiles; tile += gridDim.x) {
    const int64_t p = tile / tiles_per_poly;
    const int64_t t0 = (tile % tiles_per_poly) * TT;
    const uint32_t* ref_in = in + p * n * L + t0 * L;
    const uint32_t* lm_in = in + p * L * n + t0;
    if (TO_LM) {
      // 16-byte loads of the contiguous reference-layout run (t0 * L words in,
      // t0 a multiple of TT, so every run starts 16-byte aligned)
      for (int k4 = threadIdx.x; k4 < per / 4; k4 += blockDim.x) {
        const uint4 v = reinterpret_cast<const uint4*>(ref_in)[k4];
        if (flat) {
          sm4[k4] = v;
          continue;
        }
        const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int k = 4 * k4 + e;
          const int t = (int)(((float)k + 0.5f) * inv), l = k - t * L;
          sm[t * ld + l] = w[e];
        }
      }
    } else {
      // the limb rows of this tile (coalesced 512-byte runs), all loads issued
      // before the shared-memory stores
      constexpr int LG = 8;   // loads in flight per thread
      const int t = threadIdx.x % TT;
      for (int lb = threadIdx.x / TT; lb < L; lb += 2 * LG) {
        uint32_t wb[LG];
        const uint32_t* src = lm_in + (int64_t)lb * n + t;
#pragma unroll
        for (int k = 0; k < LG; ++k)
          if (lb + 2 * k < L) wb[k] = src[(int64_t)(2 * k) * n];
#pragma unroll
        for (int k = 0; k < LG; ++k)
          if (lb + 2 * k < L) sm[t * ld + lb + 2 * k] = wb[k];
      }
    }
    __syncthreads();
    if (TO_LM) {
      uint32_t* o = out + p * L * n + t0;
      for (int l = threadIdx.x / TT; l < L; l += blockDim.x / TT) o[(int64_t)l * n + threadIdx.x % TT] = sm[(threadIdx.x % TT) * ld + l];
    } else {
      uint32_t* o = out + p * n * L + t0 * L;
      for (int k4 = threadIdx.x; k4 < per / 4; k4 += blockDim.x) {
        if (flat) {
          reinterpret_cast<uint4*>(o)[k4] = sm4[k4];
          continue;
        }
        uint32_t w[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int k = 4 * k4 + e;
          const int t = (int)(((float)k + 0.5f) * inv), l = k - t * L;
          w[e] = sm[t * ld + l];
        }
        reinterpret_cast<uint4*>(o)[k4] = make_uint4(w[0], w[1], w[2], w[3]);
      }
    }
    __syncthreads();
  }
}

// y = Barrett(x * tab[row]) over strided limb-polynomials, 4 words per thread.
__global__ void k_modmul_table_lm(LP x, LPo y, int64_t lps, int slots, int64_t n,
                                  const uint32_t* __restrict__ tab, const uint16_t* __restrict__ trow,
                                  const ModC* __restrict__ mods, const uint16_t* __restrict__ midx) {
  const int64_t nv = n >> 2;
  for (int64_t lp = blockIdx.y; lp < lps; lp += gridDim.y) {
    const int64_t poly = lp / slots;
    const int slot = (int)(lp % slots);
    const ModC mc = mods[midx[slot]];
    const uint4* xs = (const uint4*)(x.p + poly * x.ps + slot * x.ss);
    uint4* ys = (uint4*)(y.p + poly * y.ps + slot * y.ss);
    const uint4* ts = (const uint4*)(tab + (size_t)trow[slot] * n);
    for (int64_t v = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; v < nv; v += (int64_t)gridDim.x * blockDim.x) {
      const uint4 a = xs[v], t = ts[v];
      uint4 o;
      o.x = barrett_any((uint64_t)a.x * t.x, mc);
      o.y = barrett_any((uint64_t)a.y * t.y, mc);
      o.z = barrett_any((uint64_t)a.z * t.z, mc);
      o.w = barrett_any((uint64_t)a.w * t.w, mc);
      ys[v] = o;
    }
  }
}

// out[lp][c][r] = in[lp][r][c] over strided limb-polynomials (32x33 tile).
__global__ void k_transpose_lp_any(LP in, LPo out, int64_t lps, int slots, int rows, int cols) {
  __shared__ uint32_t tile[32][33];
  const int c0 = blockIdx.x * 32, r0 = blockIdx.y * 32;
  for (int64_t lp = blockIdx.z; lp < lps; lp += gridDim.z) {
    const uint32_t* src = in.p + (lp / slots) * in.ps + (lp % slots) * in.ss;
    uint32_t* dst = out.p + (lp / slots) * out.ps + (lp % slots) * out.ss;
    for (int i = threadIdx.y; i < 32; i += blockDim.y) {
      const int r = r0 + i, c = c0 + threadIdx.x;
      if (r < rows && c < cols) tile[i][threadIdx.x] = src[(int64_t)r * cols + c];
    }
    __syncthreads();
    for (int i = threadIdx.y; i < 32; i += blockDim.y) {
      const int c = c0 + i, r = r0 + threadIdx.x;
      if (r < rows && c < cols) dst[(int64_t)c * rows + r] = tile[threadIdx.x][i];
    }
    __syncthreads();
  }
}

// Position-wise EpiOp applied in place (the CUDA-core counterpart of the
// tensor-core epilogue).
__global__ void k_apply_epi(Epi e, LPo out, int64_t lps, int slots, int64_t n, const uint16_t* __restrict__ limbs,
                            const ModC* __restrict__ mods) {
  for (int64_t lp = blockIdx.y; lp < lps; lp += gridDim.y) {
    const int64_t poly = lp / slots;
    const int slot = (int)(lp % slots);
    const ModC mc = mods[limbs[slot]];
    const uint32_t q = (uint32_t)mc.q;
    uint32_t* o = out.p + poly * out.ps + slot * out.ss;
    const uint32_t* tab = e.op == EPI_MUL ? e.tab + (int64_t)e.trow[slot] * n : nullptr;
    const uint32_t* x = (e.op == EPI_COMBINE || e.op == EPI_MODDOWN) ? e.x.at(poly, slot) : nullptr;
    const bool add_base = e.op == EPI_MODDOWN && ((e.base_mask >> (poly % e.base.E)) & 1u);
    const uint32_t* b = add_base ? e.base.at(poly, slot) : nullptr;
    const uint64_t scal = (e.op == EPI_COMBINE || e.op == EPI_MODDOWN) ? e.scal[slot] : 0;
    for (int64_t t = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; t < n; t += (int64_t)gridDim.x * blockDim.x) {
      uint32_t r = o[t];
      if (e.op == EPI_MUL) {
        r = barrett_any((uint64_t)r * tab[t], mc);
      } else if (e.op == EPI_COMBINE) {
        r = barrett_any((uint64_t)x[t] * scal + r, mc);
      } else if (e.op == EPI_MODDOWN) {
        const uint32_t sub = x[t] < r ? x[t] + q - r : x[t] - r;
        const uint32_t tt = barrett_any((uint64_t)sub * scal, mc);
        if (add_base) {
          const uint32_t s2 = b[t] + tt;
          r = s2 >= q ? s2 - q : s2;
        } else {
          r = tt;
        }
      }
      o[t] = r;
    }
  }
}

}  // namespace

int transpose_u32(const uint32_t* in, uint32_t* out, int64_t batch, int64_t rows, int64_t cols,
                  cudaStream_t st) {
  if (batch == 0 || rows == 0 || cols == 0) return CROSS_OK;
  if ((rows + 31) / 32 > 65535 || (cols + 31) / 32 > (int64_t)1 << 30) {
    set_error("transpose: %lld x %lld matrix exceeds the launch grid", (long long)rows, (long long)cols);
    return CROSS_ERR_UNSUPPORTED;
  }
  // (P, N, L) <-> (P, L, N) with few limbs: the coalesced tile kernel
  // (16-byte accesses on the contiguous side need 16-byte aligned buffers)
  const bool al = (((uintptr_t)in | (uintptr_t)out) & 15) == 0;
  const bool to_lm = al && cols <= TT_MAX_L && rows % TT == 0, to_ref = al && rows <= TT_MAX_L && cols % TT == 0;
  if (to_lm || to_ref) {
    const int64_t n = to_lm ? rows : cols;
    const int L = (int)(to_lm ? cols : rows);
    const int64_t tiles = batch * (n / TT);
    const int blocks = device_sm_count() * 8;
    const unsigned grid = (unsigned)(tiles < blocks ? tiles : blocks);
    const size_t smem = (size_t)TT * (L + 1) * sizeof(uint32_t);
    if (to_lm)
      k_transpose_ref<true><<<grid, 256, smem, st>>>(in, out, n, L, tiles);
    else
      k_transpose_ref<false><<<grid, 256, smem, st>>>(in, out, n, L, tiles);
    count_launch();
    CROSS_CHECK_CUDA(cudaGetLastError());
    return CROSS_OK;
  }
  dim3 blk(32, 8);
  for (int64_t b0 = 0; b0 < batch; b0 += 65535) {
    const int64_t nb = batch - b0 < 65535 ? batch - b0 : 65535;
    dim3 grd((unsigned)((cols + 31) / 32), (unsigned)((rows + 31) / 32), (unsigned)nb);
    k_transpose<<<grd, blk, 0, st>>>(in + b0 * rows * cols, out + b0 * rows * cols, rows, cols); count_launch();
  }
  CROSS_CHECK_CUDA(cudaGetLastError());
  return CROSS_OK;
}

int transpose_lp(LP in, LPo out, int64_t polys, int slots, int rows, int cols, cudaStream_t st) {
  const int64_t lps = polys * slots;
  if (lps == 0) return CROSS_OK;
  if ((rows + 31) / 32 > 65535) {
    set_error("transpose_lp: %d rows exceed the launch grid", rows);
    return CROSS_ERR_UNSUPPORTED;
  }
  dim3 blk(32, 8), grd((unsigned)((cols + 31) / 32), (unsigned)((rows + 31) / 32), (unsigned)(lps < 65535 ? lps : 65535));
  k_transpose_lp_any<<<grd, blk, 0, st>>>(in, out, lps, slots, rows, cols);
  count_launch();
  CROSS_CHECK_CUDA(cudaGetLastError());
  return CROSS_OK;
}

int apply_epi(const Epi& e, LPo out, int64_t polys, int slots, int64_t N, const uint16_t* limbs, const ModC* mods,
              cudaStream_t st) {
  const int64_t lps = polys * slots;
  if (e.op == EPI_NONE || lps == 0) return CROSS_OK;
  unsigned gx = (unsigned)((N + EW_THREADS - 1) / EW_THREADS);
  if (gx > 64) gx = 64;
  k_apply_epi<<<dim3(gx, (unsigned)(lps < 65535 ? lps : 65535)), EW_THREADS, 0, st>>>(e, out, lps, slots, N, limbs, mods);
  count_launch();
  CROSS_CHECK_CUDA(cudaGetLastError());
  return CROSS_OK;
}

int modmul_table_lm(LP x, LPo y, int64_t polys, int slots, int64_t n, const uint32_t* tab,
                    const uint16_t* trow, const ModC* mods, const uint16_t* midx, cudaStream_t st) {
  const int64_t lps = polys * slots;
  if (lps == 0) return CROSS_OK;
  if (n % 4) {
    set_error("modmul_table_lm: n=%lld must be a multiple of 4", (long long)n);
    return CROSS_ERR_UNSUPPORTED;
  }
  const int64_t nv = n / 4;
  unsigned gx = (unsigned)((nv + EW_THREADS - 1) / EW_THREADS);
  if (gx > 64) gx = 64;
  dim3 grd(gx, (unsigned)(lps < 65535 ? lps : 65535));
  k_modmul_table_lm<<<grd, EW_THREADS, 0, st>>>(x, y, lps, slots, n, tab, trow, mods, midx); count_launch();
  CROSS_CHECK_CUDA(cudaGetLastError());
  return CROSS_OK;
}

}  // namespace cross

using namespace cross;

extern "C" {

int cross_mod_reduce(cross_moduli mods, const void* in, int in_is_u64, uint32_t* out, int64_t rows,
                     void* stream) {
  CROSS_REQUIRE(mods && rows >= 0 && (rows == 0 || (in && out)), "cross_mod_reduce: bad argument");
  const int64_t total = rows * mods->n;
  if (total == 0) return CROSS_OK;
  const cudaStream_t st = (cudaStream_t)stream;
  if (total < EW32_LIMIT) {
    if (in_is_u64)
      k_mod_reduce32<true><<<ew_blocks(total, 4), EW_THREADS, 0, st>>>(in, out, (uint32_t)total, mods->n, mods->dev);
    else
      k_mod_reduce32<false><<<ew_blocks(total, 4), EW_THREADS, 0, st>>>(in, out, (uint32_t)total, mods->n, mods->dev);
  } else if (in_is_u64) {
    k_mod_reduce<true><<<ew_blocks(total, 4), EW_THREADS, 0, st>>>(in, out, total, mods->n, mods->dev);
  } else {
    k_mod_reduce<false><<<ew_blocks(total, 4), EW_THREADS, 0, st>>>(in, out, total, mods->n, mods->dev);
  }
  count_launch();
  CROSS_CHECK_CUDA(cudaGetLastError());
  return CROSS_OK;
}

int cross_mod_reduce_ex(cross_moduli mods, int reduction, const uint64_t* z, const uint64_t* z_s, void* out,
                        int64_t rows, void* stream) {
  CROSS_REQUIRE(mods && rows >= 0 && (rows == 0 || (z && out)), "cross_mod_reduce_ex: bad argument");
  CROSS_REQUIRE(reduction != CROSS_REDUCTION_SHOUP || rows == 0 || z_s,
                "cross_mod_reduce_ex: Shoup's reduction needs z_s");
  if (reduction == CROSS_REDUCTION_BARRETT) return cross_mod_reduce(mods, z, 1, (uint32_t*)out, rows, stream);
  const int64_t total = rows * mods->n;
  if (total == 0) return CROSS_OK;
  cudaStream_t st = (cudaStream_t)stream;
  switch (reduction) {
    case CROSS_REDUCTION_MONTGOMERY:
      k_mod_reduce_var<CROSS_REDUCTION_MONTGOMERY><<<ew_blocks(total, 4), EW_THREADS, 0, st>>>(z, z_s, out, total,
                                                                                               mods->n, mods->dev_v);
      break;
    case CROSS_REDUCTION_SHOUP:
      k_mod_reduce_var<CROSS_REDUCTION_SHOUP><<<ew_blocks(total, 4), EW_THREADS, 0, st>>>(z, z_s, out, total, mods->n,
                                                                                          mods->dev_v);
      break;
    case CROSS_REDUCTION_BAT_LAZY:
      k_mod_reduce_var<CROSS_REDUCTION_BAT_LAZY><<<ew_blocks(total, 4), EW_THREADS, 0, st>>>(z, z_s, out, total,
                                                                                             mods->n, mods->dev_v);
      break;
    default:
      set_error("cross_mod_reduce_ex: unknown reduction %d", reduction);
      return CROSS_ERR_INVALID_ARG;
  }
  count_launch();
  CROSS_CHECK_CUDA(cudaGetLastError());
  return CROSS_OK;
}

int cross_modmul(cross_moduli mods, const void* a, int a_is_u64, const void* b, int b_is_u64,
                 int64_t b_rows, uint32_t* out, int64_t rows, void* stream) {
  CROSS_REQUIRE(mods && rows >= 0 && b_rows >= 1 && (rows == 0 || (a && b && out)), "cross_modmul: bad argument");
  const int64_t total = rows * mods->n;
  if (total == 0) return CROSS_OK;
  const cudaStream_t st = (cudaStream_t)stream;
  if (total < EW32_LIMIT) {
    const int64_t bm = b_rows >= rows ? 0 : b_rows * mods->n;
    const unsigned g = ew_blocks(total, 4);
    const uint32_t t32 = (uint32_t)total, M = (uint32_t)mods->n;
    if (!a_is_u64 && !b_is_u64 && total % 4 == 0 && bm % 4 == 0 && aligned16(a) && aligned16(b) && aligned16(out)) {
      const auto* a32 = static_cast<const uint32_t*>(a);
      const auto* b32 = static_cast<const uint32_t*>(b);
      const unsigned gv = ew_blocks(total / 4, 1);
      if (bm)
        k_modmul32v<true><<<gv, EW_THREADS, 0, st>>>(a32, b32, (uint32_t)bm, out, t32 / 4, M, mods->dev, mods->dev_f);
      else
        k_modmul32v<false><<<gv, EW_THREADS, 0, st>>>(a32, b32, 0u, out, t32 / 4, M, mods->dev, mods->dev_f);
    } else if (a_is_u64 && b_is_u64) {
      k_modmul32<true, true><<<g, EW_THREADS, 0, st>>>(a, b, (uint32_t)bm, out, t32, M, mods->dev);
    } else if (a_is_u64) {
      k_modmul32<true, false><<<g, EW_THREADS, 0, st>>>(a, b, (uint32_t)bm, out, t32, M, mods->dev);
    } else if (b_is_u64) {
      k_modmul32<false, true><<<g, EW_THREADS, 0, st>>>(a, b, (uint32_t)bm, out, t32, M, mods->dev);
    } else {
      k_modmul32<false, false><<<g, EW_THREADS, 0, st>>>(a, b, (uint32_t)bm, out, t32, M, mods->dev);
    }
  } else {
    k_modmul_ref<<<ew_blocks(total, 4), EW_THREADS, 0, st>>>(a, a_is_u64, b, b_is_u64, b_rows, out, total, mods->n,
                                                          mods->dev);
  }
  count_launch();
  CROSS_CHECK_CUDA(cudaGetLastError());
  return CROSS_OK;
}

int cross_tensor_product(cross_moduli mods, const uint32_t* ct, uint32_t* out01, uint32_t* out2,
                         int64_t batch, int64_t n, void* stream) {
  CROSS_REQUIRE(mods && batch >= 0 && n >= 0 && (batch == 0 || n == 0 || (ct && out01 && out2)),
                "cross_tensor_product: bad argument");
  const int64_t per = n * mods->n;
  if (batch * per == 0) return CROSS_OK;
  k_tensor_ref<<<ew_blocks(batch * per, 4), EW_THREADS, 0, (cudaStream_t)stream>>>(ct, out01, out2, batch, per,
                                                                                  mods->n, mods->dev); count_launch();
  CROSS_CHECK_CUDA(cudaGetLastError());
  return CROSS_OK;
}

int cross_add_mod(cross_moduli mods, const uint32_t* a, const uint32_t* b, uint32_t* out, int64_t elements,
                  int64_t n, void* stream) {
  CROSS_REQUIRE(mods && elements >= 0 && n >= 0 && (elements == 0 || n == 0 || (a && b && out)),
                "cross_add_mod: bad argument");
  const int64_t total = elements * mods->n * n;
  if (total == 0) return CROSS_OK;
  if (total < EW32_LIMIT && n % 4 == 0 && aligned16(a) && aligned16(b) && aligned16(out))
    k_add_mod32v<<<ew_blocks(total / 4, 1), EW_THREADS, 0, (cudaStream_t)stream>>>(
        a, b, out, (uint32_t)(total / 4), (uint32_t)n, log2_or_neg(n), mods->n, mods->dev);
  else if (total < EW32_LIMIT)
    k_add_mod32<<<ew_blocks(total, 4), EW_THREADS, 0, (cudaStream_t)stream>>>(a, b, out, (uint32_t)total, (uint32_t)n,
                                                                             log2_or_neg(n), mods->n, mods->dev);
  else
    k_add_mod<<<ew_blocks(total, 4), EW_THREADS, 0, (cudaStream_t)stream>>>(a, b, out, total, n, mods->n, mods->dev);
  count_launch();
  CROSS_CHECK_CUDA(cudaGetLastError());
  return CROSS_OK;
}

int cross_automorphism(const uint32_t* in, const int32_t* coef_map, uint32_t* out, int64_t polys, int64_t n,
                       int num_limbs, void* stream) {
  CROSS_REQUIRE(polys >= 0 && n > 0 && num_limbs > 0 && (polys == 0 || (in && coef_map && out && in != out)),
                "cross_automorphism: bad argument (in and out must differ)");
  const int64_t total = polys * n * num_limbs;
  if (total == 0) return CROSS_OK;
  if (total < EW32_LIMIT)
    k_gather_rows32<<<ew_blocks(total, 4), EW_THREADS, 0, (cudaStream_t)stream>>>(
        in, coef_map, out, (uint32_t)total, (uint32_t)n, log2_or_neg(n), (uint32_t)num_limbs);
  else
    k_gather_rows<<<ew_blocks(total, 4), EW_THREADS, 0, (cudaStream_t)stream>>>(in, coef_map, out, polys, n, num_limbs);
  count_launch();
  CROSS_CHECK_CUDA(cudaGetLastError());
  return CROSS_OK;
}

int cross_to_limb_major(const uint32_t* in, uint32_t* out, int64_t polys, int64_t n, int num_limbs,
                        void* stream) {
  CROSS_REQUIRE(polys >= 0 && n > 0 && num_limbs > 0 && (polys == 0 || (in && out && in != out)),
                "cross_to_limb_major: bad argument (in and out must differ)");
  return transpose_u32(in, out, polys, n, num_limbs, (cudaStream_t)stream);
}

int cross_to_reference(const uint32_t* in, uint32_t* out, int64_t polys, int64_t n, int num_limbs,
                       void* stream) {
  CROSS_REQUIRE(polys >= 0 && n > 0 && num_limbs > 0 && (polys == 0 || (in && out && in != out)),
                "cross_to_reference: bad argument (in and out must differ)");
  return transpose_u32(in, out, polys, num_limbs, n, (cudaStream_t)stream);
}

}  // extern "C"
