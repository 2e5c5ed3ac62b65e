// BAT matrix NTT / INTT (ntt_mm.py:351-407) -- plan creation and the
// CUDA-core kernels used for every size (dp4a contractions; the tcgen05
// tensor-core path in ntt_tc.cu takes over for the large factorisations).
//
// The 3-step NTT of one limb-polynomial, viewed as an R x C matrix X:
//   step 1 ("col"):  S1[z,c] = sum_{r,q} byte_q(X[r,c]) * T1bat[z,q,r,p] << 8p
//                    Y = Barrett(Barrett(S1) * T2)                  (ntt_mm.py:372-375)
//   step 3 ("row"):  S3[z,n] = sum_{c,q} byte_q(Y[z,c]) * T3bat[c,q,n,p] << 8p
//                    out = Barrett(S3)                               (ntt_mm.py:376-377)
// and the INTT is the row transform (with the intt_tf_step2 twiddle) followed
// by the column transform (ntt_mm.py:401-406).  Sums are exact integers, so any
// exact evaluation order reproduces the reference bit for bit.
#include <cstdlib>
#include <cstring>
#include <vector>

#include "internal.hpp"

namespace cross {

namespace {

constexpr int TM = 16;   // output rows per block
constexpr int TN = 64;   // output cols per block
constexpr int TK = 32;   // contraction chunk

// Reductions of one output: step 1 (+ step 2 when TWIDDLE) or step 3 of
// ntt_mm.py:372-377 with the plan's reduction (RedMode): Barrett, Montgomery
// (every reduction, ntt_mm.py:432-440), or BAT-lazy (step 1 lazy in uint64,
// the step-2 product in uint64 with wrap-around, Barrett after; ntt_mm.py:602-630).
template <bool TWIDDLE, int RED>
__device__ __forceinline__ uint32_t stage_reduce(uint64_t z, const ModC& mc, const VarC& vc, uint32_t tw) {
  if (RED == RED_MONTGOMERY) {
    const uint32_t v = montgomery(z, vc.q, vc.qinv);
    return TWIDDLE ? montgomery((uint64_t)v * tw, vc.q, vc.qinv) : v;
  }
  if (RED == RED_BAT_LAZY && TWIDDLE) return barrett_any(bat_lazy(z, vc.r) * tw, mc);
  const uint32_t v = barrett_any(z, mc);
  return TWIDDLE ? barrett_any((uint64_t)v * tw, mc) : v;
}

// Column transform: out[z, c] = epi( sum_k W[z, k] (.) X[k, c] ), k over R.
template <bool TWIDDLE, int RED>
__global__ void __launch_bounds__(256) k_col_dp4a(LP in, LPo out, int64_t lps, int slots,
                                                  const uint16_t* __restrict__ limbs, int R, int C,
                                                  const uint32_t* __restrict__ W,
                                                  const uint32_t* __restrict__ T2,
                                                  const ModC* __restrict__ mods,
                                                  const VarC* __restrict__ varc) {
  __shared__ uint32_t Xs[TK][TN + 4];
  __shared__ uint32_t Ws[4][TM][TK + 1];
  const int tid = threadIdx.x, tx = tid & 15, ty = tid >> 4;
  const int c0 = blockIdx.x * TN, z0 = blockIdx.y * TM;
  for (int64_t lp = blockIdx.z; lp < lps; lp += gridDim.z) {
    const int64_t poly = lp / slots;
    const int slot = (int)(lp % slots);
    const int limb = limbs[slot];
    const uint32_t* x = in.p + poly * in.ps + slot * in.ss;
    uint32_t* y = out.p + poly * out.ps + slot * out.ss;
    const uint32_t* w = W + (size_t)limb * 4 * R * R;
    uint32_t acc[4][4];
#pragma unroll
    for (int j = 0; j < 4; ++j)
#pragma unroll
      for (int p = 0; p < 4; ++p) acc[j][p] = 0;
    for (int k0 = 0; k0 < R; k0 += TK) {
      for (int i = tid; i < TK * TN; i += 256) {
        const int k = i / TN, cc = i % TN;
        const int gk = k0 + k, gc = c0 + cc;
        Xs[k][cc] = (gk < R && gc < C) ? x[(size_t)gk * C + gc] : 0u;
      }
      for (int i = tid; i < 4 * TM * TK; i += 256) {
        const int p = i / (TM * TK), zz = (i / TK) % TM, k = i % TK;
        const int gz = z0 + zz, gk = k0 + k;
        Ws[p][zz][k] = (gz < R && gk < R) ? w[((size_t)p * R + gz) * R + gk] : 0u;
      }
      __syncthreads();
#pragma unroll 4
      for (int k = 0; k < TK; ++k) {
        const uint32_t a0 = Ws[0][ty][k], a1 = Ws[1][ty][k], a2 = Ws[2][ty][k], a3 = Ws[3][ty][k];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const uint32_t b = Xs[k][tx * 4 + j];
          acc[j][0] = __dp4a(b, a0, acc[j][0]);
          acc[j][1] = __dp4a(b, a1, acc[j][1]);
          acc[j][2] = __dp4a(b, a2, acc[j][2]);
          acc[j][3] = __dp4a(b, a3, acc[j][3]);
        }
      }
      __syncthreads();
    }
    const int z = z0 + ty;
    if (z < R) {
      const ModC mc = mods[limb];
      VarC vc{};
      if (RED >= RED_MONTGOMERY) vc = varc[limb];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int cc = c0 + tx * 4 + j;
        if (cc < C) {
          const uint32_t tw = TWIDDLE ? T2[((size_t)limb * R + z) * C + cc] : 0u;
          y[(size_t)z * C + cc] =
              stage_reduce<TWIDDLE, RED>(combine4(acc[j][0], acc[j][1], acc[j][2], acc[j][3]), mc, vc, tw);
        }
      }
    }
  }
}

// Row transform: out[r, n] = epi( sum_k X[r, k] (.) U[k, n] ), k over C.
template <bool TWIDDLE, int RED>
__global__ void __launch_bounds__(256) k_row_dp4a(LP in, LPo out, int64_t lps, int slots,
                                                  const uint16_t* __restrict__ limbs, int R, int C,
                                                  const uint32_t* __restrict__ U,
                                                  const uint32_t* __restrict__ T2,
                                                  const ModC* __restrict__ mods,
                                                  const VarC* __restrict__ varc) {
  __shared__ uint32_t Xs[TM][TK + 1];
  __shared__ uint32_t Us[4][TK][TN + 4];
  const int tid = threadIdx.x, tx = tid & 15, ty = tid >> 4;
  const int n0 = blockIdx.x * TN, r0 = blockIdx.y * TM;
  for (int64_t lp = blockIdx.z; lp < lps; lp += gridDim.z) {
    const int64_t poly = lp / slots;
    const int slot = (int)(lp % slots);
    const int limb = limbs[slot];
    const uint32_t* x = in.p + poly * in.ps + slot * in.ss;
    uint32_t* y = out.p + poly * out.ps + slot * out.ss;
    const uint32_t* u = U + (size_t)limb * 4 * C * C;
    uint32_t acc[4][4];
#pragma unroll
    for (int j = 0; j < 4; ++j)
#pragma unroll
      for (int p = 0; p < 4; ++p) acc[j][p] = 0;
    for (int k0 = 0; k0 < C; k0 += TK) {
      for (int i = tid; i < TM * TK; i += 256) {
        const int rr = i / TK, k = i % TK;
        const int gr = r0 + rr, gk = k0 + k;
        Xs[rr][k] = (gr < R && gk < C) ? x[(size_t)gr * C + gk] : 0u;
      }
      for (int i = tid; i < 4 * TK * TN; i += 256) {
        const int p = i / (TK * TN), k = (i / TN) % TK, nn = i % TN;
        const int gk = k0 + k, gn = n0 + nn;
        Us[p][k][nn] = (gk < C && gn < C) ? u[((size_t)p * C + gk) * C + gn] : 0u;
      }
      __syncthreads();
#pragma unroll 4
      for (int k = 0; k < TK; ++k) {
        const uint32_t a = Xs[ty][k];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          acc[j][0] = __dp4a(a, Us[0][k][tx * 4 + j], acc[j][0]);
          acc[j][1] = __dp4a(a, Us[1][k][tx * 4 + j], acc[j][1]);
          acc[j][2] = __dp4a(a, Us[2][k][tx * 4 + j], acc[j][2]);
          acc[j][3] = __dp4a(a, Us[3][k][tx * 4 + j], acc[j][3]);
        }
      }
      __syncthreads();
    }
    const int r = r0 + ty;
    if (r < R) {
      const ModC mc = mods[limb];
      VarC vc{};
      if (RED >= RED_MONTGOMERY) vc = varc[limb];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int nn = n0 + tx * 4 + j;
        if (nn < C) {
          const uint32_t tw = TWIDDLE ? T2[((size_t)limb * R + r) * C + nn] : 0u;
          y[(size_t)r * C + nn] =
              stage_reduce<TWIDDLE, RED>(combine4(acc[j][0], acc[j][1], acc[j][2], acc[j][3]), mc, vc, tw);
        }
      }
    }
  }
}

// Pack the reference's (X, 4 q, Y, 4 p, M) u8 BAT array into
// dst[m][p][row][col] u32 (4 q-bytes per word).  `transpose_xy` selects
// whether the first BAT axis (X) is the output row (col transforms: [z][k]) or
// the contraction row (row transforms: [k][n]).
// Every limb's output is written in order and each word once; the M limbs of
// one source position are read together (contiguous in the source).
void pack_bat(const uint8_t* bat, int X, int Y, int M, std::vector<uint32_t>& dst) {
  dst.resize((size_t)M * 4 * X * Y);
  const size_t lw = (size_t)4 * X * Y;     // words per limb
  const size_t qs = (size_t)Y * 4 * M;     // source stride of q
  for (int p = 0; p < 4; ++p)
    for (int x = 0; x < X; ++x)
      for (int y = 0; y < Y; ++y) {
        const uint8_t* s = bat + (((size_t)x * 4 * Y + y) * 4 + p) * M;
        uint32_t* d = dst.data() + ((size_t)p * X + x) * Y + y;
        for (int m = 0; m < M; ++m)
          d[m * lw] = (uint32_t)s[m] | (uint32_t)s[qs + m] << 8 | (uint32_t)s[2 * qs + m] << 16 |
                      (uint32_t)s[3 * qs + m] << 24;
      }
}

void unpack_tw(const uint32_t* tw, int R, int C, int M, std::vector<uint32_t>& dst) {
  dst.resize((size_t)M * R * C);
  for (int r = 0; r < R; ++r)
    for (int c = 0; c < C; ++c)
      for (int m = 0; m < M; ++m) dst[((size_t)m * R + r) * C + c] = tw[((size_t)r * C + c) * M + m];
}

unsigned grid_z(int64_t lps) { return (unsigned)(lps < 65535 ? lps : 65535); }

}  // namespace

int64_t ntt_tmp_words(const cross_ntt_plan_s* P, int64_t lps) { return lps * P->r * P->c * 2; }

static int ntt_run_dp4a(const cross_ntt_plan_s* P, bool inverse, LP in, LPo out, int64_t polys, int slots,
                        const uint16_t* limbs, uint32_t* tmp, cudaStream_t st);

int ntt_run(const cross_ntt_plan_s* P, bool inverse, LP in, LPo out, int64_t polys, int slots,
            const uint16_t* limbs, uint32_t* tmp, cudaStream_t st) {
  return ntt_exec(P, inverse, in, COEF_NATURAL, out, COEF_NATURAL, polys, slots, limbs, Epi{}, tmp, st);
}

int ntt_exec(const cross_ntt_plan_s* P, bool inverse, LP in, int in_layout, LPo out, int out_layout, int64_t polys,
             int slots, const uint16_t* limbs, const Epi& epi, uint32_t* tmp, cudaStream_t st) {
  const int64_t lps = polys * slots;
  if (lps == 0) return CROSS_OK;
  if (P->tc) return ntt_exec_tc(P, inverse, in, in_layout, out, out_layout, polys, slots, limbs, epi, tmp, st);
  if (P->tc64 && in_layout == COEF_NATURAL && out_layout == COEF_NATURAL && epi.op == EPI_NONE &&
      (((uintptr_t)in.p | (uintptr_t)out.p) & 15) == 0 && in.ps % 4 == 0 && in.ss % 4 == 0 && out.ps % 4 == 0 &&
      out.ss % 4 == 0)
    return ntt64_run(P, inverse, in, out, polys, slots, limbs, st);
  // CUDA-core path: natural-order transforms composed with the layout
  // conversions and the position-wise op.
  auto run = P->red == CROSS_REDUCTION_SHOUP ? ntt_run_shoup : ntt_run_dp4a;
  const int R = P->r, C = P->c;
  const int64_t N = (int64_t)R * C;
  uint32_t* t2 = tmp + lps * N;
  int rc;
  if (!inverse) {
    LP src = in;
    if (in_layout == COEF_TRANSPOSED) {
      if ((rc = transpose_lp(in, LPo{t2, slots * N, N}, polys, slots, C, R, st))) return rc;
      src = LP{t2, slots * N, N};
    }
    if ((rc = run(P, false, src, out, polys, slots, limbs, tmp, st))) return rc;
  } else if (out_layout == COEF_NATURAL) {
    if ((rc = run(P, true, in, out, polys, slots, limbs, tmp, st))) return rc;
  } else {
    if ((rc = run(P, true, in, LPo{t2, slots * N, N}, polys, slots, limbs, tmp, st))) return rc;
    if ((rc = transpose_lp(LP{t2, slots * N, N}, out, polys, slots, R, C, st))) return rc;
  }
  return apply_epi(epi, out, polys, slots, N, limbs, P->mods, st);
}

template <int RED>
static int run_dp4a(const cross_ntt_plan_s* P, bool inverse, LP in, LPo out, LPo mid, LP mid_in, int64_t lps, int slots,
                    const uint16_t* limbs, cudaStream_t st) {
  const int R = P->r, C = P->c;
  dim3 blk(256);
  dim3 g((C + TN - 1) / TN, (R + TM - 1) / TM, grid_z(lps));
  if (!inverse) {
    k_col_dp4a<true, RED><<<g, blk, 0, st>>>(in, mid, lps, slots, limbs, R, C, P->col_fwd, P->tw_fwd, P->mods, P->varc);
    count_launch();
    k_row_dp4a<false, RED><<<g, blk, 0, st>>>(mid_in, out, lps, slots, limbs, R, C, P->row_fwd, nullptr, P->mods, P->varc);
    count_launch();
  } else {
    k_row_dp4a<true, RED><<<g, blk, 0, st>>>(in, mid, lps, slots, limbs, R, C, P->row_inv, P->tw_inv, P->mods, P->varc);
    count_launch();
    k_col_dp4a<false, RED><<<g, blk, 0, st>>>(mid_in, out, lps, slots, limbs, R, C, P->col_inv, nullptr, P->mods, P->varc);
    count_launch();
  }
  CROSS_CHECK_CUDA(cudaGetLastError());
  return CROSS_OK;
}

static int ntt_run_dp4a(const cross_ntt_plan_s* P, bool inverse, LP in, LPo out, int64_t polys, int slots,
                        const uint16_t* limbs, uint32_t* tmp, cudaStream_t st) {
  const int R = P->r, C = P->c;
  const int64_t N = (int64_t)R * C;
  const int64_t lps = polys * slots;
  if (lps == 0) return CROSS_OK;
  LPo mid{tmp, (int64_t)slots * N, N};
  LP mid_in{tmp, (int64_t)slots * N, N};
  switch (P->red) {
    case CROSS_REDUCTION_MONTGOMERY:
      return run_dp4a<RED_MONTGOMERY>(P, inverse, in, out, mid, mid_in, lps, slots, limbs, st);
    case CROSS_REDUCTION_BAT_LAZY:
      return run_dp4a<RED_BAT_LAZY>(P, inverse, in, out, mid, mid_in, lps, slots, limbs, st);
    default:
      return run_dp4a<RED_BARRETT>(P, inverse, in, out, mid, mid_in, lps, slots, limbs, st);
  }
}

// Plan fields shared by every reduction: sizes, moduli, identity limb map and,
// for Montgomery / BAT-lazy, the per-limb VarC.  On failure *out is freed.
static int plan_base(cross_moduli moduli, int r, int c, int red, cross_ntt_plan_s** out) {
  const int M = moduli->n;
  auto* P = new cross_ntt_plan_s();
  *out = P;
  P->r = r;
  P->c = c;
  P->M = M;
  P->red = red;
  P->mods_host = moduli->host;
  std::vector<uint16_t> ident(M);
  for (int i = 0; i < M; ++i) ident[i] = (uint16_t)i;
  int rc = upload_vec(&P->mods, P->mods_host);
  if (!rc) rc = upload_vec(&P->identity, ident);
  if (!rc && (red == CROSS_REDUCTION_MONTGOMERY || red == CROSS_REDUCTION_BAT_LAZY))
    rc = upload_vec(&P->varc, make_varc(P->mods_host));
  return rc;
}

}  // namespace cross

using namespace cross;

extern "C" {

int cross_ntt_plan_create_ex(cross_moduli moduli, int r, int c, int reduction, const uint8_t* ntt_bat_tf_step1,
                             const uint32_t* ntt_tf_step2, const uint8_t* ntt_bat_tf_step3,
                             const uint8_t* intt_bat_tf_step1, const uint32_t* intt_tf_step2,
                             const uint8_t* intt_bat_tf_step3, cross_ntt_plan* out) {
  CROSS_REQUIRE(out && moduli && ntt_bat_tf_step1 && ntt_tf_step2 && ntt_bat_tf_step3 &&
                    intt_bat_tf_step1 && intt_tf_step2 && intt_bat_tf_step3,
                "cross_ntt_plan_create: null argument");
  CROSS_REQUIRE(r >= 1 && c >= 1 && r <= 4096 && c <= 4096,
                "cross_ntt_plan_create: r=%d c=%d out of range", r, c);
  CROSS_REQUIRE(reduction == CROSS_REDUCTION_BARRETT || reduction == CROSS_REDUCTION_MONTGOMERY ||
                    reduction == CROSS_REDUCTION_BAT_LAZY,
                "cross_ntt_plan_create_ex: reduction %d needs another table set (Shoup: "
                "cross_ntt_plan_create_shoup)", reduction);
  *out = nullptr;
  cross_ntt_plan_s* P = nullptr;
  int rc = plan_base(moduli, r, c, reduction, &P);
  const int M = moduli->n;
  std::vector<uint32_t> buf;
  if (!rc) { pack_bat(ntt_bat_tf_step1, r, r, M, buf); rc = upload_vec(&P->col_fwd, buf); }
  if (!rc) { pack_bat(intt_bat_tf_step3, r, r, M, buf); rc = upload_vec(&P->col_inv, buf); }
  if (!rc) { pack_bat(ntt_bat_tf_step3, c, c, M, buf); rc = upload_vec(&P->row_fwd, buf); }
  if (!rc) { pack_bat(intt_bat_tf_step1, c, c, M, buf); rc = upload_vec(&P->row_inv, buf); }
  if (!rc) { unpack_tw(ntt_tf_step2, r, c, M, buf); rc = upload_vec(&P->tw_fwd, buf); }
  if (!rc) { unpack_tw(intt_tf_step2, r, c, M, buf); rc = upload_vec(&P->tw_inv, buf); }
  // CROSS_B200_DISABLE_TC=1 keeps the CUDA-core contraction for every size (a
  // diagnostic for comparing the two exact implementations).
  const char* no_tc = getenv("CROSS_B200_DISABLE_TC");
  if (!rc && !(no_tc && no_tc[0] == '1'))
    rc = tc_plan_init(P, ntt_bat_tf_step1, ntt_bat_tf_step3, intt_bat_tf_step1, intt_bat_tf_step3, intt_tf_step2);
  if (rc) {
    cross_ntt_plan_destroy(P);
    return rc;
  }
  *out = P;
  return CROSS_OK;
}

int cross_ntt_plan_create(cross_moduli moduli, int r, int c, const uint8_t* ntt_bat_tf_step1,
                          const uint32_t* ntt_tf_step2, const uint8_t* ntt_bat_tf_step3,
                          const uint8_t* intt_bat_tf_step1, const uint32_t* intt_tf_step2,
                          const uint8_t* intt_bat_tf_step3, cross_ntt_plan* out) {
  return cross_ntt_plan_create_ex(moduli, r, c, CROSS_REDUCTION_BARRETT, ntt_bat_tf_step1, ntt_tf_step2,
                                  ntt_bat_tf_step3, intt_bat_tf_step1, intt_tf_step2, intt_bat_tf_step3, out);
}

int cross_ntt_plan_create_shoup(cross_moduli moduli, int r, int c, const uint32_t* const* tables,
                                cross_ntt_plan* out) {
  CROSS_REQUIRE(out && moduli && tables, "cross_ntt_plan_create_shoup: null argument");
  for (int i = 0; i < 12; ++i) CROSS_REQUIRE(tables[i], "cross_ntt_plan_create_shoup: table %d is null", i);
  CROSS_REQUIRE(r >= 1 && c >= 1 && r <= 4096 && c <= 4096,
                "cross_ntt_plan_create_shoup: r=%d c=%d out of range", r, c);
  *out = nullptr;
  cross_ntt_plan_s* P = nullptr;
  int rc = plan_base(moduli, r, c, CROSS_REDUCTION_SHOUP, &P);
  // (X, Y, M) host tables -> [M][X][Y]
  const int dims[6][2] = {{r, r}, {r, c}, {c, c}, {c, c}, {r, c}, {r, r}};
  std::vector<uint32_t> buf;
  for (int i = 0; i < 6 && !rc; ++i) {
    unpack_tw(tables[i], dims[i][0], dims[i][1], P->M, buf);
    rc = upload_vec(&P->sh[i], buf);
    if (!rc) {
      unpack_tw(tables[6 + i], dims[i][0], dims[i][1], P->M, buf);
      rc = upload_vec(&P->sh_s[i], buf);
    }
  }
  if (rc) {
    cross_ntt_plan_destroy(P);
    return rc;
  }
  *out = P;
  return CROSS_OK;
}

int cross_ntt_plan_reduction(cross_ntt_plan P) {
  CROSS_REQUIRE(P, "cross_ntt_plan_reduction: null plan");
  return P->red;
}

int cross_ntt_plan_check(cross_ntt_plan P) {
  CROSS_REQUIRE(P, "cross_ntt_plan_check: null plan");
  if (!P->tc_err) return CROSS_OK;
  int code = 0;
  CROSS_CHECK_CUDA(cudaDeviceSynchronize());
  CROSS_CHECK_CUDA(cudaMemcpy(&code, P->tc_err, sizeof(int), cudaMemcpyDeviceToHost));
  if (!code) return CROSS_OK;
  const int zero = 0;
  CROSS_CHECK_CUDA(cudaMemcpy(P->tc_err, &zero, sizeof(int), cudaMemcpyHostToDevice));
  set_error("tensor-core NTT kernel: a bounded wait expired (role code %d)", code);
  return CROSS_ERR_TIMEOUT;
}

int cross_ntt_plan_destroy(cross_ntt_plan P) {
  if (!P) return CROSS_OK;
  dfree(P->mods);
  dfree(P->identity);
  dfree(P->col_fwd);
  dfree(P->col_inv);
  dfree(P->row_fwd);
  dfree(P->row_inv);
  dfree(P->tw_fwd);
  dfree(P->tw_inv);
  dfree(P->varc);
  for (int i = 0; i < 6; ++i) {
    dfree(P->sh[i]);
    dfree(P->sh_s[i]);
  }
  tc_plan_free(P);
  delete P;
  return CROSS_OK;
}

size_t cross_ntt_workspace_size(cross_ntt_plan P, int64_t batch, int layout) {
  if (!P || batch < 0) return 0;
  const size_t words = (size_t)batch * P->M * P->r * P->c;
  Arena a(nullptr, 0);
  a.take<uint32_t>((size_t)ntt_tmp_words(P, batch * P->M));
  if (layout == CROSS_LAYOUT_REFERENCE) a.take<uint32_t>(words);
  return a.off;
}

int cross_ntt(cross_ntt_plan P, int inverse, const uint32_t* in, uint32_t* out, int64_t batch, int layout,
              void* workspace, size_t workspace_bytes, void* stream) {
  CROSS_REQUIRE(P && batch >= 0 && (batch == 0 || (in && out)), "cross_ntt: null argument or negative batch");
  CROSS_REQUIRE(layout == CROSS_LAYOUT_REFERENCE || layout == CROSS_LAYOUT_LIMB_MAJOR ||
                    layout == CROSS_LAYOUT_LIMB_MAJOR_TRANSPOSED,
                "cross_ntt: unknown layout %d", layout);
  if (batch == 0) return CROSS_OK;
  const size_t need = cross_ntt_workspace_size(P, batch, layout);
  if (!workspace || workspace_bytes < need) {
    set_error("cross_ntt: workspace of %zu bytes required, %zu given", need, workspace_bytes);
    return CROSS_ERR_WORKSPACE;
  }
  cudaStream_t st = (cudaStream_t)stream;
  const int64_t N = (int64_t)P->r * P->c;
  const int M = P->M;
  const size_t words = (size_t)batch * M * N;
  Arena a(workspace, workspace_bytes);
  uint32_t* tmp = a.take<uint32_t>((size_t)ntt_tmp_words(P, batch * M));
  if (layout == CROSS_LAYOUT_LIMB_MAJOR) {
    return ntt_run(P, inverse != 0, LP{in, M * N, N}, LPo{out, M * N, N}, batch, M, P->identity, tmp, st);
  }
  if (layout == CROSS_LAYOUT_LIMB_MAJOR_TRANSPOSED) {
    return ntt_exec(P, inverse != 0, LP{in, M * N, N}, COEF_TRANSPOSED, LPo{out, M * N, N}, COEF_TRANSPOSED, batch, M,
                    P->identity, Epi{}, tmp, st);
  }
  uint32_t* lm = a.take<uint32_t>(words);
  int rc = transpose_u32(in, lm, batch, N, M, st);
  if (rc) return rc;
  rc = ntt_run(P, inverse != 0, LP{lm, M * N, N}, LPo{lm, M * N, N}, batch, M, P->identity, tmp, st);
  if (rc) return rc;
  return transpose_u32(lm, out, batch, M, N, st);
}

}  // extern "C"
