// Basis conversion with the Montgomery, Shoup and BAT-lazy contexts
// (bconv.py:261-390), on the CUDA cores.
//
// Per coefficient t of a polynomial, with x_i the source limbs:
//   step 1  c_i from x_i * QHatInvModq_i (uint64):
//     Montgomery  c_i = Mont_i(x_i QHatInvModq_i)                       (bconv.py:273, 234-244)
//                 basis_change only: c_i = (c_i 2^-32 mod q_i) 2^32 mod p_{i'} (bconv.py:275-280),
//                 i' = i (size_q == size_p) or 0 (size_p == 1), the reference's broadcast
//     Shoup       c_i = (uint32)(x_i QHatInvModq_i - ((x_i QHatInvModq_shoup_i) >> 32) q_i) (bconv.py:325-327)
//     BAT-lazy    basis_change      c_i = Lazy_i(x_i QHatInvModq_i) mod q_i          (bconv.py:351-355)
//                 basis_change_bat  c_i = ((uint32)Lazy_i(x_i QHatInvModq_i)) mod q_i (bconv.py:382-386)
//   step 2  per target limb j:
//     basis_change      z_j = sum_i c_i QHatModp[i][j] (uint64, wrapping); Shoup also
//                       z_s,j = sum_i c_i QHatModp_shoup[i][j]               (bconv.py:282-287, 329-337)
//     basis_change_bat  z_j = sum_b (sum_{i,a} byte_a(c_i) QHatModpBAT[(i,a), j, b]) << 8b (bconv.py:246)
//   step 3  Montgomery: Mont_j(z_j) (uint32); Shoup: (uint32)(z_j - (z_s,j >> 32) p_j);
//           BAT-lazy: Lazy_j(z_j) (uint64)                                    (bconv.py:288, 338, 368)
#include <type_traits>

#include "internal.hpp"

namespace cross {

namespace {

constexpr int BV_THREADS = 128;

template <int RED, bool BAT, int SQMAX>
__global__ void __launch_bounds__(BV_THREADS) k_bconv_var(const uint32_t* __restrict__ in, int64_t in_ps,
                                                          int64_t in_ls, int64_t in_ts, void* __restrict__ out,
                                                          int64_t out_ps, int64_t out_ls, int64_t out_ts,
                                                          int64_t polys, int64_t n, int sq, int sp,
                                                          const VarC* __restrict__ src, const VarC* __restrict__ dst,
                                                          const uint32_t* __restrict__ qhat_inv,
                                                          const uint32_t* __restrict__ qhat_inv_s,
                                                          const uint32_t* __restrict__ tab,
                                                          const uint32_t* __restrict__ tab_s) {
  // tables in shared memory: BAT [sp][4][sq] packed over the 4 source bytes,
  // else [sp][sq] (and the Shoup companion [sp][sq] after it)
  extern __shared__ uint32_t ts[];
  const int tabn = BAT ? sp * 4 * sq : sp * sq;
  for (int i = threadIdx.x; i < tabn; i += BV_THREADS) ts[i] = tab[i];
  if (RED == CROSS_REDUCTION_SHOUP)
    for (int i = threadIdx.x; i < sp * sq; i += BV_THREADS) ts[tabn + i] = tab_s[i];
  __syncthreads();
  const int64_t total = polys * n;
  for (int64_t e = (int64_t)blockIdx.x * BV_THREADS + threadIdx.x; e < total; e += (int64_t)gridDim.x * BV_THREADS) {
    const int64_t poly = e / n, t = e - poly * n;
    const uint32_t* x = in + poly * in_ps + t * in_ts;
    uint32_t c[SQMAX];
#pragma unroll
    for (int i = 0; i < SQMAX; ++i) {
      if (i >= sq) break;
      const VarC s = src[i];
      const uint32_t xv = x[i * in_ls];
      const uint64_t cu = (uint64_t)xv * qhat_inv[i];
      uint32_t ci;
      if (RED == CROSS_REDUCTION_MONTGOMERY) {
        ci = montgomery(cu, s.q, s.qinv);
        if (!BAT) {
          const uint64_t back = ((uint64_t)ci * s.winv) % s.q;
          const uint32_t p = dst[sp == 1 ? 0 : i].q;
          ci = (uint32_t)((back << 32) % p);
        }
      } else if (RED == CROSS_REDUCTION_SHOUP) {
        ci = shoup((uint32_t)cu, __umulhi(xv, qhat_inv_s[i]), s.q);
      } else {
        const uint64_t l = bat_lazy(cu, s.r);
        ci = BAT ? (uint32_t)l % s.q : (uint32_t)(l % s.q);
      }
      c[i] = ci;
    }
    for (int j = 0; j < sp; ++j) {
      const VarC d = dst[j];
      uint64_t z = 0, zs = 0;
      if (BAT) {
        uint32_t acc[4] = {0, 0, 0, 0};
        const uint32_t* tj = ts + (size_t)j * 4 * sq;
#pragma unroll
        for (int i = 0; i < SQMAX; ++i) {
          if (i >= sq) break;
#pragma unroll
          for (int b = 0; b < 4; ++b) acc[b] = __dp4a(c[i], tj[b * sq + i], acc[b]);
        }
        z = combine4(acc[0], acc[1], acc[2], acc[3]);
      } else {
        const uint32_t* tj = ts + (size_t)j * sq;
        const uint32_t* tsj = ts + tabn + (size_t)j * sq;
#pragma unroll
        for (int i = 0; i < SQMAX; ++i) {
          if (i >= sq) break;
          z += (uint64_t)c[i] * tj[i];
          if (RED == CROSS_REDUCTION_SHOUP) zs += (uint64_t)c[i] * tsj[i];
        }
      }
      const int64_t o = poly * out_ps + j * out_ls + t * out_ts;
      if (RED == CROSS_REDUCTION_BAT_LAZY)
        static_cast<uint64_t*>(out)[o] = bat_lazy(z, d.r);
      else if (RED == CROSS_REDUCTION_MONTGOMERY)
        static_cast<uint32_t*>(out)[o] = montgomery(z, d.q, d.qinv);
      else
        static_cast<uint32_t*>(out)[o] = shoup((uint32_t)z, (uint32_t)(zs >> 32), d.q);
    }
  }
}

template <int RED, bool BAT, int SQMAX>
int launch_var(const cross_bconv_plan_s* P, const uint32_t* in, int64_t in_ps, int64_t in_ls, int64_t in_ts,
               void* out, int64_t out_ps, int64_t out_ls, int64_t out_ts, int64_t polys, int64_t n, cudaStream_t st) {
  const int sq = P->sq, sp = P->sp;
  const size_t words = BAT ? (size_t)sp * 4 * sq : (size_t)sp * sq * (RED == CROSS_REDUCTION_SHOUP ? 2 : 1);
  const size_t smem = words * sizeof(uint32_t);
  auto kern = k_bconv_var<RED, BAT, SQMAX>;
  CROSS_CHECK_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
  const int64_t blocks = (polys * n + BV_THREADS - 1) / BV_THREADS;
  const int64_t cap = (int64_t)device_sm_count() * 8;
  kern<<<(unsigned)(blocks < cap ? blocks : cap), BV_THREADS, smem, st>>>(
      in, in_ps, in_ls, in_ts, out, out_ps, out_ls, out_ts, polys, n, sq, sp, P->src_v, P->dst_v, P->qhat_inv,
      P->qhat_inv_s, BAT ? P->bat : P->qhat_modp, P->qhat_modp_s);
  count_launch();
  CROSS_CHECK_CUDA(cudaGetLastError());
  return CROSS_OK;
}

template <int RED, bool BAT>
int launch_var_sq(const cross_bconv_plan_s* P, const uint32_t* in, int64_t in_ps, int64_t in_ls, int64_t in_ts,
                  void* out, int64_t out_ps, int64_t out_ls, int64_t out_ts, int64_t polys, int64_t n,
                  cudaStream_t st) {
  if (P->sq <= 8) return launch_var<RED, BAT, 8>(P, in, in_ps, in_ls, in_ts, out, out_ps, out_ls, out_ts, polys, n, st);
  if (P->sq <= 32)
    return launch_var<RED, BAT, 32>(P, in, in_ps, in_ls, in_ts, out, out_ps, out_ls, out_ts, polys, n, st);
  return launch_var<RED, BAT, 64>(P, in, in_ps, in_ls, in_ts, out, out_ps, out_ls, out_ts, polys, n, st);
}

}  // namespace

int bconv_var_run(const cross_bconv_plan_s* P, bool bat, const uint32_t* in, int64_t in_ps, int64_t in_ls,
                  int64_t in_ts, void* out, int64_t out_ps, int64_t out_ls, int64_t out_ts, int64_t polys,
                  int64_t n, cudaStream_t st) {
  if (polys == 0 || n == 0) return CROSS_OK;
  if (P->sq > 64 || (size_t)P->sp * 4 * P->sq * sizeof(uint32_t) > 200 * 1024) {
    set_error("bconv: size_q=%d size_p=%d exceed the supported tile (size_q <= 64)", P->sq, P->sp);
    return CROSS_ERR_UNSUPPORTED;
  }
#define CROSS_BV(RED)                                                                                          \
  return bat ? launch_var_sq<RED, true>(P, in, in_ps, in_ls, in_ts, out, out_ps, out_ls, out_ts, polys, n, st) \
             : launch_var_sq<RED, false>(P, in, in_ps, in_ls, in_ts, out, out_ps, out_ls, out_ts, polys, n, st)
  if (bat && (P->red == CROSS_REDUCTION_MONTGOMERY || P->red == CROSS_REDUCTION_BAT_LAZY)) {
    // the tensor-core contraction when the shape allows, else the CUDA cores
    const int rc = bconv_var_tc(P, in, in_ps, in_ls, in_ts, out, out_ps, out_ls, out_ts, polys, n, st);
    if (rc != CROSS_ERR_UNSUPPORTED) return rc;
  }
  switch (P->red) {
    case CROSS_REDUCTION_MONTGOMERY:
      if (!bat && P->sq != P->sp && P->sp != 1) {
        set_error("bconv (Montgomery) basis_change: source limbs are re-encoded with the target modulus of the "
                  "same index (bconv.py:278-280), so size_q (%d) must equal size_p (%d) or size_p must be 1",
                  P->sq, P->sp);
        return CROSS_ERR_INVALID_ARG;
      }
      CROSS_BV(CROSS_REDUCTION_MONTGOMERY);
    case CROSS_REDUCTION_SHOUP:
      if (bat) {
        set_error("bconv (Shoup): basis_change_bat calls the two-operand Shoup reduction with one operand "
                  "(bconv.py:244); only basis_change is defined");
        return CROSS_ERR_UNSUPPORTED;
      }
      return launch_var_sq<CROSS_REDUCTION_SHOUP, false>(P, in, in_ps, in_ls, in_ts, out, out_ps, out_ls, out_ts,
                                                          polys, n, st);
    case CROSS_REDUCTION_BAT_LAZY:
      CROSS_BV(CROSS_REDUCTION_BAT_LAZY);
    default:
      set_error("bconv: plan reduction %d has no variant kernel", P->red);
      return CROSS_ERR_INVALID_ARG;
  }
#undef CROSS_BV
}

}  // namespace cross
