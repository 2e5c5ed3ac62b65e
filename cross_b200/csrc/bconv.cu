// Basis conversion (bconv.py:173-252).
//
// basis_change_bat: c_i = Barrett_src_i(x_i * QHatInvModq_i); then for every
// target limb j the BAT contraction
//   S_j = sum_b ( sum_{i,a} byte_a(c_i) * QHatModpBAT[(i,a), j, b] ) << 8b
// and out_j = Barrett_dst_j(S_j).  The inner sum over the four bytes a of one
// c_i is one dp4a against the packed BAT column.
// basis_change: S_j = sum_i c_i * QHatModp[i, j] in uint64, then Barrett.
#include <type_traits>
#include <vector>

#include "internal.hpp"

namespace cross {

namespace {

constexpr int BC_THREADS = 128;
constexpr int BC_COEF = 4;   // coefficients per thread

// Each thread converts BC_COEF consecutive coefficients of one polynomial: the
// source residues c_i = Barrett(x_i * QHatInvModq_i) stay in registers, so each
// shared-memory table word feeds BC_COEF dp4a (BAT) or multiply-adds.
template <int SQMAX, bool BAT, bool VEC>
__global__ void __launch_bounds__(BC_THREADS) k_bconv(const uint32_t* __restrict__ in, int64_t in_ps,
                                                      int64_t in_ls, int64_t in_ts, uint32_t* __restrict__ out,
                                                      int64_t out_ps, int64_t out_ls, int64_t out_ts,
                                                      int64_t polys, int64_t n, int sq, int sp,
                                                      const ModC* __restrict__ src, const ModC* __restrict__ dst,
                                                      const uint32_t* __restrict__ qhat_inv,
                                                      const uint32_t* __restrict__ tab,
                                                      const uint32_t* __restrict__ twist,
                                                      const uint16_t* __restrict__ trow) {
  extern __shared__ uint32_t ts[];   // BAT: [sp][4][sq], else [sp][sq]
  const int tabn = BAT ? sp * 4 * sq : sp * sq;
  for (int i = threadIdx.x; i < tabn; i += BC_THREADS) ts[i] = tab[i];
  __syncthreads();
  const int64_t per_block = (int64_t)BC_THREADS * BC_COEF;
  const int64_t tiles = (n + per_block - 1) / per_block;
  for (int64_t w = blockIdx.x; w < polys * tiles; w += gridDim.x) {
    const int64_t poly = w / tiles;
    const int64_t t0 = (w % tiles) * per_block + (int64_t)threadIdx.x * BC_COEF;
    if (t0 >= n) continue;
    const int nc = (int)(n - t0 < BC_COEF ? n - t0 : BC_COEF);
    const uint32_t* x = in + poly * in_ps + t0 * in_ts;
    uint32_t c[BC_COEF][SQMAX];
#pragma unroll
    for (int i = 0; i < SQMAX; ++i) {
      if (i < sq) {
        const ModC mc = src[i];
        const uint64_t qi = qhat_inv[i];
        uint32_t xv[BC_COEF];
        if (VEC) {
          const uint4 v = *reinterpret_cast<const uint4*>(x + i * in_ls);
          xv[0] = v.x; xv[1] = v.y; xv[2] = v.z; xv[3] = v.w;
        } else {
#pragma unroll
          for (int k = 0; k < BC_COEF; ++k) xv[k] = k < nc ? x[i * in_ls + k * in_ts] : 0u;
        }
#pragma unroll
        for (int k = 0; k < BC_COEF; ++k) c[k][i] = barrett_any((uint64_t)xv[k] * qi, mc);
      }
    }
    uint32_t* y = out + poly * out_ps + t0 * out_ts;
    for (int j = 0; j < sp; ++j) {
      const ModC mc = dst[j];
      uint32_t r[BC_COEF];
      if (BAT) {
        uint32_t acc[4][BC_COEF];
#pragma unroll
        for (int b = 0; b < 4; ++b)
#pragma unroll
          for (int k = 0; k < BC_COEF; ++k) acc[b][k] = 0;
        const uint32_t* tj = ts + (size_t)j * 4 * sq;
#pragma unroll
        for (int i = 0; i < SQMAX; ++i) {
          if (i < sq) {
#pragma unroll
            for (int b = 0; b < 4; ++b) {
              const uint32_t tw = tj[b * sq + i];
#pragma unroll
              for (int k = 0; k < BC_COEF; ++k) acc[b][k] = __dp4a(c[k][i], tw, acc[b][k]);
            }
          }
        }
#pragma unroll
        for (int k = 0; k < BC_COEF; ++k) r[k] = barrett_any(combine4(acc[0][k], acc[1][k], acc[2][k], acc[3][k]), mc);
      } else {
        uint64_t acc[BC_COEF] = {};
        const uint32_t* tj = ts + (size_t)j * sq;
#pragma unroll
        for (int i = 0; i < SQMAX; ++i) {
          if (i < sq) {
            const uint64_t tw = tj[i];
#pragma unroll
            for (int k = 0; k < BC_COEF; ++k) acc[k] += (uint64_t)c[k][i] * tw;
          }
        }
#pragma unroll
        for (int k = 0; k < BC_COEF; ++k) r[k] = barrett_any(acc[k], mc);
      }
      if (twist) {
        const uint32_t* tw = twist + (int64_t)trow[j] * n + t0;
#pragma unroll
        for (int k = 0; k < BC_COEF; ++k)
          if (k < nc) r[k] = barrett_any((uint64_t)r[k] * tw[k], mc);
      }
      if (VEC) {
        *reinterpret_cast<uint4*>(y + j * out_ls) = make_uint4(r[0], r[1], r[2], r[3]);
      } else {
#pragma unroll
        for (int k = 0; k < BC_COEF; ++k)
          if (k < nc) y[j * out_ls + k * out_ts] = r[k];
      }
    }
  }
}

template <int SQMAX, bool BAT>
int launch_bconv(const cross_bconv_plan_s* P, bool vec, const uint32_t* in, int64_t in_ps, int64_t in_ls,
                 int64_t in_ts, uint32_t* out, int64_t out_ps, int64_t out_ls, int64_t out_ts, int64_t polys,
                 int64_t n, cudaStream_t st, const uint32_t* twist, const uint16_t* trow) {
  const size_t smem = (size_t)P->sp * (BAT ? 4 : 1) * P->sq * sizeof(uint32_t);
  const int64_t work = polys * ((n + BC_THREADS * BC_COEF - 1) / (BC_THREADS * BC_COEF));
  const unsigned grid = (unsigned)(work < 148 * 8 ? work : 148 * 8);
  const uint32_t* tab = BAT ? P->bat : P->qhat_modp;
  if (vec) {
    CROSS_CHECK_CUDA(cudaFuncSetAttribute(k_bconv<SQMAX, BAT, true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                          (int)smem));
    k_bconv<SQMAX, BAT, true><<<grid, BC_THREADS, smem, st>>>(in, in_ps, in_ls, in_ts, out, out_ps, out_ls, out_ts,
                                                              polys, n, P->sq, P->sp, P->src, P->dst, P->qhat_inv,
                                                              tab, twist, trow);
  } else {
    CROSS_CHECK_CUDA(cudaFuncSetAttribute(k_bconv<SQMAX, BAT, false>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                          (int)smem));
    k_bconv<SQMAX, BAT, false><<<grid, BC_THREADS, smem, st>>>(in, in_ps, in_ls, in_ts, out, out_ps, out_ls, out_ts,
                                                               polys, n, P->sq, P->sp, P->src, P->dst, P->qhat_inv,
                                                               tab, twist, trow);
  }
  count_launch();
  CROSS_CHECK_CUDA(cudaGetLastError());
  return CROSS_OK;
}

}  // namespace

int bconv_run(const cross_bconv_plan_s* P, bool bat, const uint32_t* in, int64_t in_ps, int64_t in_ls,
              int64_t in_ts, uint32_t* out, int64_t out_ps, int64_t out_ls, int64_t out_ts, int64_t polys,
              int64_t n, cudaStream_t st, const uint32_t* twist, const uint16_t* trow) {
  if (polys == 0 || n == 0) return CROSS_OK;
  const size_t smem = (size_t)P->sp * 4 * P->sq * sizeof(uint32_t);
  if (smem > 200 * 1024 || P->sq > 64) {
    set_error("bconv: size_q=%d size_p=%d exceed the supported tile (size_q <= 64)", P->sq, P->sp);
    return CROSS_ERR_UNSUPPORTED;
  }
  // 16-byte vector access when coefficients are contiguous and every row is aligned
  const bool vec = in_ts == 1 && out_ts == 1 && n % BC_COEF == 0 && (((uintptr_t)in | (uintptr_t)out) & 15) == 0 &&
                   in_ps % 4 == 0 && in_ls % 4 == 0 && out_ps % 4 == 0 && out_ls % 4 == 0;
  const int sqmax = P->sq <= 8 ? 8 : P->sq <= 16 ? 16 : P->sq <= 32 ? 32 : 64;
  auto go = [&](auto sqm) {
    constexpr int S = decltype(sqm)::value;
    return bat ? launch_bconv<S, true>(P, vec, in, in_ps, in_ls, in_ts, out, out_ps, out_ls, out_ts, polys, n, st,
                                       twist, trow)
               : launch_bconv<S, false>(P, vec, in, in_ps, in_ls, in_ts, out, out_ps, out_ls, out_ts, polys, n, st,
                                        twist, trow);
  };
  switch (sqmax) {
    case 8: return go(std::integral_constant<int, 8>{});
    case 16: return go(std::integral_constant<int, 16>{});
    case 32: return go(std::integral_constant<int, 32>{});
    default: return go(std::integral_constant<int, 64>{});
  }
}

}  // namespace cross

using namespace cross;

extern "C" {

int cross_bconv_plan_create(cross_moduli src, cross_moduli dst, const uint32_t* qhat_inv_modq,
                            const uint32_t* qhat_modp, const uint8_t* qhat_modp_bat, cross_bconv_plan* out) {
  CROSS_REQUIRE(src && dst && qhat_inv_modq && qhat_modp && qhat_modp_bat && out,
                "cross_bconv_plan_create: null argument");
  *out = nullptr;
  auto* P = new cross_bconv_plan_s();
  P->sq = src->n;
  P->sp = dst->n;
  P->src_host = src->host;
  P->dst_host = dst->host;
  const int sq = P->sq, sp = P->sp;
  std::vector<uint32_t> bat((size_t)sp * 4 * sq, 0u), qm((size_t)sp * sq);
  // qhat_modp_bat[(i*4 + a), j, b] (bconv.py:93-97) -> bat[j][b][i] packed over a.
  for (int i = 0; i < sq; ++i)
    for (int a = 0; a < 4; ++a)
      for (int j = 0; j < sp; ++j)
        for (int b = 0; b < 4; ++b)
          bat[((size_t)j * 4 + b) * sq + i] |= (uint32_t)qhat_modp_bat[(((size_t)i * 4 + a) * sp + j) * 4 + b] << (8 * a);
  for (int i = 0; i < sq; ++i)
    for (int j = 0; j < sp; ++j) qm[(size_t)j * sq + i] = qhat_modp[(size_t)i * sp + j];
  std::vector<uint32_t> qi(qhat_inv_modq, qhat_inv_modq + sq);
  int rc = upload_vec(&P->src, P->src_host);
  if (!rc) rc = upload_vec(&P->dst, P->dst_host);
  if (!rc) rc = upload_vec(&P->qhat_inv, qi);
  if (!rc) rc = upload_vec(&P->bat, bat);
  if (!rc) rc = upload_vec(&P->qhat_modp, qm);
  if (rc) {
    cross_bconv_plan_destroy(P);
    return rc;
  }
  *out = P;
  return CROSS_OK;
}

int cross_bconv_plan_destroy(cross_bconv_plan P) {
  if (!P) return CROSS_OK;
  dfree(P->src);
  dfree(P->dst);
  dfree(P->qhat_inv);
  dfree(P->bat);
  dfree(P->qhat_modp);
  delete P;
  return CROSS_OK;
}

int cross_bconv(cross_bconv_plan P, int bat, const uint32_t* in, uint32_t* out, int64_t batch, int64_t n,
                int layout, void* stream) {
  CROSS_REQUIRE(P && in && out && in != out && batch >= 0 && n >= 0, "cross_bconv: bad argument");
  const int sq = P->sq, sp = P->sp;
  if (layout == CROSS_LAYOUT_REFERENCE)
    return bconv_run(P, bat != 0, in, n * sq, 1, sq, out, n * sp, 1, sp, batch, n, (cudaStream_t)stream);
  CROSS_REQUIRE(layout == CROSS_LAYOUT_LIMB_MAJOR, "cross_bconv: unknown layout %d", layout);
  return bconv_run(P, bat != 0, in, n * sq, n, 1, out, n * sp, n, 1, batch, n, (cudaStream_t)stream);
}

}  // extern "C"
