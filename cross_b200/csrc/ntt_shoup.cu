// Shoup-reduction NTT / INTT (ntt_mm.py:443-587, ntt_sm.py:415-494) on the
// CUDA cores.
//
// The reference evaluates each matrix product of the 3-step transform as a
// byte convolution recombined in uint64 (ntt_mm.py:40-65), which is the exact
// sum of the uint32 x uint32 products modulo 2^64, and reduces it with
// ShoupContext.modular_reduction against the same product taken with the
// companion table floor(T 2^32 / q), cast to uint32:
//     out = (uint32)(z - (z_s >> 32) q),  z = sum T x,  z_s = sum T_s x.
// Only the low word of z and bits 32..63 of z_s reach the result, so a thread
// accumulates z in uint32 and z_s in uint64.  Step 2 multiplies elementwise by
// the step-2 table the same way (ntt_mm.py:534-537):
//     out2 = (uint32)(r T2 - ((r T2_s) >> 32) q).
// Stages, for one limb-polynomial X (R x C, row-major):
//   ntt   Z = T1 X (table on the left), Z *= T2, W = Z T3 (table on the right)
//   intt  Y = X iT1 (right), Y *= iT2, V = iT3 Y (left)
#include "internal.hpp"

namespace cross {

namespace {

constexpr int SH_T = 64;    // output tile edge
constexpr int SH_K = 16;    // contraction chunk

// out[m][n] = reduce(sum_k A[m][k] B[k][n]) for every limb-polynomial; the
// table (and its companion) is A when TAB_A (rows x K per limb), else B
// (K x cols per limb); the data operand is the other one.  Output rows x cols.
template <bool TAB_A, bool TW>
__global__ void __launch_bounds__(256) k_shoup_stage(LP in, LPo out, int64_t lps, int slots,
                                                     const uint16_t* __restrict__ limbs, int rows, int cols, int K,
                                                     const uint32_t* __restrict__ T, const uint32_t* __restrict__ Ts,
                                                     const uint32_t* __restrict__ T2,
                                                     const uint32_t* __restrict__ T2s,
                                                     const ModC* __restrict__ mods) {
  __shared__ uint32_t As[SH_K][SH_T + 1];   // [k][m]
  __shared__ uint32_t Bs[SH_K][SH_T + 1];   // [k][n]
  __shared__ uint32_t Cs[SH_K][SH_T + 1];   // companion tile, on the table's side
  const int tid = threadIdx.x, tx = tid & 15, ty = tid >> 4;
  const int n0 = blockIdx.x * SH_T, m0 = blockIdx.y * SH_T;
  for (int64_t lp = blockIdx.z; lp < lps; lp += gridDim.z) {
    const int64_t poly = lp / slots;
    const int slot = (int)(lp % slots);
    const int limb = limbs[slot];
    const uint32_t* x = in.p + poly * in.ps + slot * in.ss;
    uint32_t* y = out.p + poly * out.ps + slot * out.ss;
    const size_t tab_words = TAB_A ? (size_t)rows * K : (size_t)K * cols;
    const uint32_t* t = T + (size_t)limb * tab_words;
    const uint32_t* ts = Ts + (size_t)limb * tab_words;
    const uint32_t* A = TAB_A ? t : x;       // rows x K
    const uint32_t* B = TAB_A ? x : t;       // K x cols
    uint32_t acc[4][4];
    uint64_t acc_s[4][4];
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        acc[i][j] = 0;
        acc_s[i][j] = 0;
      }
    for (int k0 = 0; k0 < K; k0 += SH_K) {
      for (int i = tid; i < SH_T * SH_K; i += 256) {
        const int mm = i / SH_K, kk = i % SH_K;
        const int gm = m0 + mm, gk = k0 + kk;
        const bool ok = gm < rows && gk < K;
        As[kk][mm] = ok ? A[(size_t)gm * K + gk] : 0u;
        if (TAB_A) Cs[kk][mm] = ok ? ts[(size_t)gm * K + gk] : 0u;
      }
      for (int i = tid; i < SH_K * SH_T; i += 256) {
        const int kk = i / SH_T, nn = i % SH_T;
        const int gk = k0 + kk, gn = n0 + nn;
        const bool ok = gk < K && gn < cols;
        Bs[kk][nn] = ok ? B[(size_t)gk * cols + gn] : 0u;
        if (!TAB_A) Cs[kk][nn] = ok ? ts[(size_t)gk * cols + gn] : 0u;
      }
      __syncthreads();
#pragma unroll 4
      for (int kk = 0; kk < SH_K; ++kk) {
        uint32_t a[4], b[4], c[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          a[i] = As[kk][ty + 16 * i];
          b[i] = Bs[kk][tx + 16 * i];
          c[i] = TAB_A ? Cs[kk][ty + 16 * i] : Cs[kk][tx + 16 * i];
        }
#pragma unroll
        for (int i = 0; i < 4; ++i)
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            acc[i][j] += a[i] * b[j];
            acc_s[i][j] += TAB_A ? (uint64_t)c[i] * b[j] : (uint64_t)a[i] * c[j];
          }
      }
      __syncthreads();
    }
    const uint32_t q = (uint32_t)mods[limb].q;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int m = m0 + ty + 16 * i;
      if (m >= rows) continue;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int n = n0 + tx + 16 * j;
        if (n >= cols) continue;
        uint32_t r = shoup(acc[i][j], (uint32_t)(acc_s[i][j] >> 32), q);
        if (TW) {
          const size_t o = ((size_t)limb * rows + m) * cols + n;
          const uint32_t w = T2[o], ws = T2s[o];
          r = shoup(r * w, __umulhi(r, ws), q);
        }
        y[(size_t)m * cols + n] = r;
      }
    }
  }
}

unsigned grid_z(int64_t lps) { return (unsigned)(lps < 65535 ? lps : 65535); }

}  // namespace

int ntt_run_shoup(const cross_ntt_plan_s* P, bool inverse, LP in, LPo out, int64_t polys, int slots,
                  const uint16_t* limbs, uint32_t* tmp, cudaStream_t st) {
  const int R = P->r, C = P->c;
  const int64_t N = (int64_t)R * C;
  const int64_t lps = polys * slots;
  if (lps == 0) return CROSS_OK;
  LPo mid{tmp, (int64_t)slots * N, N};
  LP mid_in{tmp, (int64_t)slots * N, N};
  const dim3 blk(256);
  const dim3 g((C + SH_T - 1) / SH_T, (R + SH_T - 1) / SH_T, grid_z(lps));
  if (!inverse) {
    // Z[z][c] = sum_r T1[z][r] X[r][c], times T2[z][c]; W[r][n] = sum_c Z[r][c] T3[c][n]
    k_shoup_stage<true, true><<<g, blk, 0, st>>>(in, mid, lps, slots, limbs, R, C, R, P->sh[0], P->sh_s[0], P->sh[1],
                                                 P->sh_s[1], P->mods);
    count_launch();
    k_shoup_stage<false, false><<<g, blk, 0, st>>>(mid_in, out, lps, slots, limbs, R, C, C, P->sh[2], P->sh_s[2],
                                                   nullptr, nullptr, P->mods);
    count_launch();
  } else {
    // Y[r][l] = sum_c X[r][c] iT1[c][l], times iT2[r][l]; V[l][c] = sum_r iT3[l][r] Y[r][c]
    k_shoup_stage<false, true><<<g, blk, 0, st>>>(in, mid, lps, slots, limbs, R, C, C, P->sh[3], P->sh_s[3], P->sh[4],
                                                  P->sh_s[4], P->mods);
    count_launch();
    k_shoup_stage<true, false><<<g, blk, 0, st>>>(mid_in, out, lps, slots, limbs, R, C, R, P->sh[5], P->sh_s[5],
                                                  nullptr, nullptr, P->mods);
    count_launch();
  }
  CROSS_CHECK_CUDA(cudaGetLastError());
  return CROSS_OK;
}

}  // namespace cross
