// Basis conversion (bconv.py:173-252).
//
// basis_change_bat: c_i = Barrett_src_i(x_i * QHatInvModq_i); then for every
// target limb j the BAT contraction
//   S_j = sum_b ( sum_{i,a} byte_a(c_i) * QHatModpBAT[(i,a), j, b] ) << 8b
// and out_j = Barrett_dst_j(S_j).  The inner sum over the four bytes a of one
// c_i is one dp4a against the packed BAT column.
// basis_change: S_j = sum_i c_i * QHatModp[i, j] in uint64, then Barrett.
#include <vector>

#include "internal.hpp"

namespace cross {

namespace {

constexpr int BC_THREADS = 128;

template <bool BAT>
__global__ void __launch_bounds__(BC_THREADS) k_bconv(const uint32_t* __restrict__ in, int64_t in_ps,
                                                      int64_t in_ls, int64_t in_ts, uint32_t* __restrict__ out,
                                                      int64_t out_ps, int64_t out_ls, int64_t out_ts,
                                                      int64_t polys, int64_t n, int sq, int sp,
                                                      const ModC* __restrict__ src, const ModC* __restrict__ dst,
                                                      const uint32_t* __restrict__ qhat_inv,
                                                      const uint32_t* __restrict__ tab,
                                                      const uint32_t* __restrict__ twist,
                                                      const uint16_t* __restrict__ trow) {
  extern __shared__ uint32_t sm[];
  uint32_t* cs = sm;                          // [sq][BC_THREADS]
  uint32_t* ts = sm + (size_t)sq * BC_THREADS;  // BAT: [sp][4][sq], else [sp][sq]
  const int tabn = BAT ? sp * 4 * sq : sp * sq;
  for (int i = threadIdx.x; i < tabn; i += BC_THREADS) ts[i] = tab[i];
  __syncthreads();
  const int64_t tiles = (n + BC_THREADS - 1) / BC_THREADS;
  for (int64_t w = blockIdx.x; w < polys * tiles; w += gridDim.x) {
    const int64_t poly = w / tiles;
    const int64_t t = (w % tiles) * BC_THREADS + threadIdx.x;
    if (t < n) {
      const uint32_t* x = in + poly * in_ps + t * in_ts;
      for (int i = 0; i < sq; ++i)
        cs[i * BC_THREADS + threadIdx.x] = barrett_any((uint64_t)x[i * in_ls] * qhat_inv[i], src[i]);
      uint32_t* y = out + poly * out_ps + t * out_ts;
      for (int j = 0; j < sp; ++j) {
        uint64_t s;
        if (BAT) {
          const uint32_t* tj = ts + (size_t)j * 4 * sq;
          uint32_t a0 = 0, a1 = 0, a2 = 0, a3 = 0;
          for (int i = 0; i < sq; ++i) {
            const uint32_t c = cs[i * BC_THREADS + threadIdx.x];
            a0 = __dp4a(c, tj[i], a0);
            a1 = __dp4a(c, tj[sq + i], a1);
            a2 = __dp4a(c, tj[2 * sq + i], a2);
            a3 = __dp4a(c, tj[3 * sq + i], a3);
          }
          s = combine4(a0, a1, a2, a3);
        } else {
          s = 0;
          const uint32_t* tj = ts + (size_t)j * sq;
          for (int i = 0; i < sq; ++i) s += (uint64_t)cs[i * BC_THREADS + threadIdx.x] * tj[i];
        }
        uint32_t r = barrett_any(s, dst[j]);
        if (twist) r = barrett_any((uint64_t)r * twist[(int64_t)trow[j] * n + t], dst[j]);
        y[j * out_ls] = r;
      }
    }
  }
}

}  // namespace

int bconv_run(const cross_bconv_plan_s* P, bool bat, const uint32_t* in, int64_t in_ps, int64_t in_ls,
              int64_t in_ts, uint32_t* out, int64_t out_ps, int64_t out_ls, int64_t out_ts, int64_t polys,
              int64_t n, cudaStream_t st, const uint32_t* twist, const uint16_t* trow) {
  if (polys == 0 || n == 0) return CROSS_OK;
  const size_t smem = ((size_t)P->sq * BC_THREADS + (size_t)P->sp * 4 * P->sq) * sizeof(uint32_t);
  if (smem > 200 * 1024) {
    set_error("bconv: size_q=%d size_p=%d exceed the shared-memory tile", P->sq, P->sp);
    return CROSS_ERR_UNSUPPORTED;
  }
  const int64_t work = polys * ((n + BC_THREADS - 1) / BC_THREADS);
  const unsigned grid = (unsigned)(work < 148 * 16 ? work : 148 * 16);
  if (bat) {
    cudaFuncSetAttribute(k_bconv<true>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    k_bconv<true><<<grid, BC_THREADS, smem, st>>>(in, in_ps, in_ls, in_ts, out, out_ps, out_ls, out_ts, polys, n,
                                                   P->sq, P->sp, P->src, P->dst, P->qhat_inv, P->bat, twist, trow); count_launch();
  } else {
    cudaFuncSetAttribute(k_bconv<false>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    k_bconv<false><<<grid, BC_THREADS, smem, st>>>(in, in_ps, in_ls, in_ts, out, out_ps, out_ls, out_ts, polys, n,
                                                    P->sq, P->sp, P->src, P->dst, P->qhat_inv, P->qhat_modp, twist, trow); count_launch();
  }
  CROSS_CHECK_CUDA(cudaGetLastError());
  return CROSS_OK;
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
