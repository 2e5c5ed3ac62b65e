// HE-Mult with relinearisation (hemul.py:153-217) and HE-Rotate
// (herot.py:183-302) as one stream of kernels over a limb-major workspace.
//
// Internal layout: every limb-polynomial is a contiguous run of N = r*c
// uint32 words; a ciphertext element is [limb][N].  The reference layout
// (..., r, c, limbs) is converted at entry and exit only.
#include <algorithm>
#include <vector>

#include "internal.hpp"
#include "tc_ptx.cuh"

namespace cross {

namespace {

constexpr int MAXPARTS = 16;
constexpr int T = 256;

struct PartPtrs {
  const uint32_t* e[MAXPARTS];   // E_j base
  int64_t ps[MAXPARTS];          // E_j poly stride (words)
};

// Barrett of finite_field.py:224-230; W32 selects the 32-bit form, exact when
// every modulus of the launch has w = 32 and m < 2^32 (plan_w32).
template <bool W32>
__device__ __forceinline__ uint32_t red(uint64_t z, const ModC& mc) {
  return W32 ? barrett_w32(z, (uint32_t)mc.q, (uint32_t)mc.m, mc.s_w) : barrett(z, mc);
}
bool plan_w32(const cross_ntt_plan_s* p) {
  for (const ModC& mc : p->mods_host)
    if (!barrett_w32_ok(mc)) return false;
  return true;
}

unsigned gx_for(int64_t nv) {
  int64_t g = (nv + T - 1) / T;
  return (unsigned)(g < 1 ? 1 : (g > 64 ? 64 : g));
}
unsigned gy_for(int64_t rows) { return (unsigned)(rows < 65535 ? rows : 65535); }

// ciphertext.py:279-295: centred lift of the last limb into every q_i,
// times gamma_i psi_i^t, Barrett.  LL: [polys][N]; out: [polys][L1][N].  A
// thread reads its four last-limb words once and writes them lifted into all
// L1 limbs (two limbs per step, table loads ahead of the arithmetic).
// FAST (every modulus passes reduce_fast_ok): the lifted word is below
// q_i + 2 q_last < 2^31 (LL is a Barrett output, below 2 q_last) and the table
// entry below q_i, so the product is below 2^31 q_i, where the 32-bit
// remainder form equals Barrett exactly.
template <bool W32, bool FAST>
__global__ void k_rescale_lift(const uint32_t* __restrict__ LL, uint32_t* __restrict__ out, int64_t polys,
                               int L1, int64_t n, uint32_t thr, uint32_t q_last,
                               const uint32_t* __restrict__ gpsi, const ModC* __restrict__ mods) {
  const int64_t nv = n >> 2;
  for (int64_t w = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; w < polys * nv;
       w += (int64_t)gridDim.x * blockDim.x) {
    const int64_t p = w / nv, v = w - p * nv;
    const uint4 x = reinterpret_cast<const uint4*>(LL + p * n)[v];
    uint4* dst = reinterpret_cast<uint4*>(out + p * L1 * n) + v;
    auto one = [&](int i, const uint4 t) {
      const ModC mc = mods[i];
      auto lift = [&](uint32_t a) -> uint64_t {
        return a < thr ? (uint64_t)a : (mc.q - (uint64_t)q_last + (uint64_t)a);
      };
      uint4 o;
      if (FAST) {
        const uint32_t q32 = (uint32_t)mc.q, m32 = (uint32_t)mc.m, sw = mc.s_w;
        auto f = [&](uint32_t a, uint32_t tv) {
          const uint32_t l = (uint32_t)lift(a);
          return tc::reduce_fast2(l * tv, __umulhi(l, tv), q32, m32, sw);
        };
        o.x = f(x.x, t.x);
        o.y = f(x.y, t.y);
        o.z = f(x.z, t.z);
        o.w = f(x.w, t.w);
      } else {
        o.x = red<W32>(lift(x.x) * t.x, mc);
        o.y = red<W32>(lift(x.y) * t.y, mc);
        o.z = red<W32>(lift(x.z) * t.z, mc);
        o.w = red<W32>(lift(x.w) * t.w, mc);
      }
      dst[(int64_t)i * (n >> 2)] = o;
    };
    int i = 0;
    for (; i + 1 < L1; i += 2) {
      const uint4 t0 = reinterpret_cast<const uint4*>(gpsi + (size_t)i * n)[v];
      const uint4 t1 = reinterpret_cast<const uint4*>(gpsi + (size_t)(i + 1) * n)[v];
      one(i, t0);
      one(i + 1, t1);
    }
    if (i < L1) one(i, reinterpret_cast<const uint4*>(gpsi + (size_t)i * n)[v]);
  }
}

// ciphertext.py:309-324 on [b][4][L1][N] -> D [b][3][L1][N].
template <bool W32>
__global__ void k_tensor_lm(const uint32_t* __restrict__ R, uint32_t* __restrict__ D, int64_t batch, int L1,
                            int64_t n, const ModC* __restrict__ mods) {
  const int64_t nv = n >> 2, rows = batch * L1, es = (int64_t)L1 * n;
  for (int64_t row = blockIdx.y; row < rows; row += gridDim.y) {
    const int64_t b = row / L1;
    const int i = (int)(row % L1);
    const ModC mc = mods[i];
    const uint32_t* base = R + b * 4 * es + (int64_t)i * n;
    uint32_t* ob = D + b * 3 * es + (int64_t)i * n;
    for (int64_t v = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; v < nv; v += (int64_t)gridDim.x * blockDim.x) {
      const uint4 a0 = ((const uint4*)base)[v], a1 = ((const uint4*)(base + es))[v];
      const uint4 b0 = ((const uint4*)(base + 2 * es))[v], b1 = ((const uint4*)(base + 3 * es))[v];
      uint4 d0, d1, d2;
#define TP(c)                                                                   \
  d0.c = red<W32>((uint64_t)a0.c * b0.c, mc);                                  \
  d1.c = red<W32>((uint64_t)a0.c * b1.c + (uint64_t)a1.c * b0.c, mc);          \
  d2.c = red<W32>((uint64_t)a1.c * b1.c, mc);
      TP(x) TP(y) TP(z) TP(w)
#undef TP
      ((uint4*)ob)[v] = d0;
      ((uint4*)(ob + es))[v] = d1;
      ((uint4*)(ob + 2 * es))[v] = d2;
    }
  }
}

// Hybrid key-switch inner product (ciphertext.py:486-518, herot.py:212-247):
// for every limb l of Q'+P, ext_j(l) is the NTT-form input limb when l is in
// digit j and the ModUp result otherwise; acc0 = sum_j ext_j * evk_b[j],
// acc1 = sum_j ext_j * evk_a[j] in uint64, then Barrett.
// Rows are walked limb-major (all ciphertexts of one limb together) so the
// limb's evaluation-key rows are read from HBM once per launch and from L2 for
// the rest of the batch.
template <bool W32, int NP>
__global__ void __launch_bounds__(128) k_ks_inner(LP dig, PartPtrs parts, const int16_t* __restrict__ src, int LT,
                                                  int64_t n, int batch, const uint32_t* __restrict__ evka,
                                                  const uint32_t* __restrict__ evkb, uint32_t* __restrict__ KS,
                                                  const ModC* __restrict__ mods) {
  // items: (limb l, ciphertext b, chunk of 128 x 4 coefficients), limb-major;
  // the host keeps their number below 2^31
  const unsigned nv = (unsigned)(n >> 2), chunks = (nv + 127) / 128;
  const unsigned items = (unsigned)batch * (unsigned)LT * chunks;
  for (unsigned it = blockIdx.x; it < items; it += gridDim.x) {
    const unsigned row = it / chunks, c = it - row * chunks;
    const int l = (int)(row / (unsigned)batch);
    const int64_t b = row - (unsigned)l * (unsigned)batch;
    const unsigned v = c * 128 + threadIdx.x;
    if (v >= nv) continue;
    uint4 e[NP], kb[NP], ka[NP];
#pragma unroll
    for (int j = 0; j < NP; ++j) {
      const int s = src[j * LT + l];
      e[j] = s < 0 ? ((const uint4*)(dig.p + b * dig.ps + (int64_t)l * dig.ss))[v]
                   : ((const uint4*)(parts.e[j] + b * parts.ps[j] + (int64_t)s * n))[v];
      kb[j] = ((const uint4*)(evkb + ((size_t)j * LT + l) * n))[v];
      ka[j] = ((const uint4*)(evka + ((size_t)j * LT + l) * n))[v];
    }
    const ModC mc = mods[l];
    uint64_t s0[4] = {0, 0, 0, 0}, s1[4] = {0, 0, 0, 0};
#pragma unroll
    for (int j = 0; j < NP; ++j) {
      s0[0] += (uint64_t)e[j].x * kb[j].x; s0[1] += (uint64_t)e[j].y * kb[j].y;
      s0[2] += (uint64_t)e[j].z * kb[j].z; s0[3] += (uint64_t)e[j].w * kb[j].w;
      s1[0] += (uint64_t)e[j].x * ka[j].x; s1[1] += (uint64_t)e[j].y * ka[j].y;
      s1[2] += (uint64_t)e[j].z * ka[j].z; s1[3] += (uint64_t)e[j].w * ka[j].w;
    }
    uint4* o0 = (uint4*)(KS + (b * 2 * LT + l) * n);
    uint4* o1 = (uint4*)(KS + (b * 2 * LT + LT + l) * n);
    o0[v] = make_uint4(red<W32>(s0[0], mc), red<W32>(s0[1], mc), red<W32>(s0[2], mc), red<W32>(s0[3], mc));
    o1[v] = make_uint4(red<W32>(s1[0], mc), red<W32>(s1[1], mc), red<W32>(s1[2], mc), red<W32>(s1[3], mc));
  }
}

// k_ks_inner for more than eight digits: one digit at a time.
template <bool W32>
__global__ void k_ks_inner_loop(LP dig, PartPtrs parts, int nparts, const int16_t* __restrict__ src, int LT,
                                int64_t n, int64_t batch, const uint32_t* __restrict__ evka,
                                const uint32_t* __restrict__ evkb, uint32_t* __restrict__ KS,
                                const ModC* __restrict__ mods) {
  const int64_t nv = n >> 2, rows = batch * LT;
  for (int64_t row = blockIdx.y; row < rows; row += gridDim.y) {
    const int l = (int)(row / batch);
    const int64_t b = row - (int64_t)l * batch;
    const ModC mc = mods[l];
    uint4* o0 = (uint4*)(KS + (b * 2 * LT + l) * n);
    uint4* o1 = (uint4*)(KS + (b * 2 * LT + LT + l) * n);
    for (int64_t v = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; v < nv; v += (int64_t)gridDim.x * blockDim.x) {
      uint64_t s0[4] = {0, 0, 0, 0}, s1[4] = {0, 0, 0, 0};
      for (int j = 0; j < nparts; ++j) {
        const int s = src[j * LT + l];
        const uint4 e = s < 0 ? ((const uint4*)(dig.p + b * dig.ps + (int64_t)l * dig.ss))[v]
                              : ((const uint4*)(parts.e[j] + b * parts.ps[j] + (int64_t)s * n))[v];
        const uint4 kb = ((const uint4*)(evkb + ((size_t)j * LT + l) * n))[v];
        const uint4 ka = ((const uint4*)(evka + ((size_t)j * LT + l) * n))[v];
        s0[0] += (uint64_t)e.x * kb.x; s0[1] += (uint64_t)e.y * kb.y;
        s0[2] += (uint64_t)e.z * kb.z; s0[3] += (uint64_t)e.w * kb.w;
        s1[0] += (uint64_t)e.x * ka.x; s1[1] += (uint64_t)e.y * ka.y;
        s1[2] += (uint64_t)e.z * ka.z; s1[3] += (uint64_t)e.w * ka.w;
      }
      o0[v] = make_uint4(red<W32>(s0[0], mc), red<W32>(s0[1], mc), red<W32>(s0[2], mc), red<W32>(s0[3], mc));
      o1[v] = make_uint4(red<W32>(s1[0], mc), red<W32>(s1[1], mc), red<W32>(s1[2], mc), red<W32>(s1[3], mc));
    }
  }
}

// Launches the key-switch inner product over batch x LT rows: the persistent
// item kernel for 2..8 digits, one block row per limb-ciphertext otherwise.
template <bool W32, int NP>
void ks_inner_items(LP dig, const PartPtrs& pp, const int16_t* src, int LT, int64_t n, int64_t B, const uint32_t* evka,
                    const uint32_t* evkb, uint32_t* KS, const ModC* mods, cudaStream_t st) {
  static PerDevice cache;   // blocks of this instantiation that fit on the GPU at once
  const int resident = cache.get([] {
    int per_sm = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, k_ks_inner<W32, NP>, 128, 0) != cudaSuccess) {
      (void)cudaGetLastError();
      per_sm = 4;
    }
    return device_sm_count() * (per_sm > 0 ? per_sm : 4);
  });
  const int64_t items = B * LT * (((n >> 2) + 127) / 128);
  const int64_t cap = resident;
  k_ks_inner<W32, NP><<<(unsigned)(items < cap ? items : cap), 128, 0, st>>>(dig, pp, src, LT, n, (int)B, evka, evkb,
                                                                           KS, mods);
}

int ks_inner(bool w32, LP dig, const PartPtrs& pp, int nparts, const int16_t* src, int LT, int64_t n, int64_t B,
             const uint32_t* evka, const uint32_t* evkb, uint32_t* KS, const ModC* mods, cudaStream_t st) {
  const int64_t items = B * LT * (((n >> 2) + 127) / 128);
  if (nparts >= 2 && nparts <= 8 && items < ((int64_t)1 << 31)) {
#define CROSS_KS(NP)                                                                              \
  (w32 ? ks_inner_items<true, NP>(dig, pp, src, LT, n, B, evka, evkb, KS, mods, st)               \
       : ks_inner_items<false, NP>(dig, pp, src, LT, n, B, evka, evkb, KS, mods, st))
    switch (nparts) {
      case 2: CROSS_KS(2); break;
      case 3: CROSS_KS(3); break;
      case 4: CROSS_KS(4); break;
      case 5: CROSS_KS(5); break;
      case 6: CROSS_KS(6); break;
      case 7: CROSS_KS(7); break;
      default: CROSS_KS(8); break;
    }
#undef CROSS_KS
  } else {
    const dim3 g(gx_for(n >> 2), gy_for(B * LT));
    if (w32)
      k_ks_inner_loop<true><<<g, T, 0, st>>>(dig, pp, nparts, src, LT, n, B, evka, evkb, KS, mods);
    else
      k_ks_inner_loop<false><<<g, T, 0, st>>>(dig, pp, nparts, src, LT, n, B, evka, evkb, KS, mods);
  }
  count_launch();
  CROSS_CHECK_CUDA(cudaGetLastError());
  return CROSS_OK;
}

// out[p][l][j] = in[p][l][map[j]] (limb-major automorphism, jnp.take semantics).
__global__ void k_gather_lm(const uint32_t* __restrict__ in, const int32_t* __restrict__ map,
                            uint32_t* __restrict__ out, int64_t rows, int64_t n) {
  for (int64_t row = blockIdx.y; row < rows; row += gridDim.y) {
    for (int64_t j = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; j < n; j += (int64_t)gridDim.x * blockDim.x) {
      int64_t s = map[j];
      if (s < 0) s += n;
      out[row * n + j] = (s < 0 || s >= n) ? 0xFFFFFFFFu : in[row * n + s];
    }
  }
}

bool same_q(const ModC& a, const ModC& b) { return a.q == b.q && a.m == b.m && a.w == b.w && a.s_w == b.s_w; }

// rows x N table, natural coefficient order -> transposed order for an (R x C)
// factorisation: out[row][c*R + r] = in[row][r*C + c].
std::vector<uint32_t> to_transposed(const uint32_t* tab, int rows, int R, int C) {
  const int64_t N = (int64_t)R * C;
  std::vector<uint32_t> out((size_t)rows * N);
  for (int row = 0; row < rows; ++row)
    for (int r = 0; r < R; ++r)
      for (int c = 0; c < C; ++c) out[(size_t)row * N + (size_t)c * R + r] = tab[(size_t)row * N + (size_t)r * C + c];
  return out;
}

// Rescale by the last prime (ciphertext.py:267-303) on `polys` limb-major
// polynomials: X has L limbs per poly (stride xps, evaluation order), R
// receives L-1 limbs (stride L1*N).  The coefficient-domain intermediates stay
// in transposed order: INTT(last limb) x psi^-i (fused) -> lift x gamma psi
// -> NTT with x*beta + y fused into its last stage.  plan covers the L moduli
// of Q at indices 0..L-1 (m_last = {L-1}, m_q1 = 0..L-2); mods_q1 are the
// Barrett constants of Q'; the two tables are in transposed order.
struct RescaleArgs {
  const cross_ntt_plan_s* ntt;
  const uint16_t* m_last;
  const uint16_t* m_zero;
  const uint16_t* m_q1;
  const ModC* mods_q1;
  const uint32_t* inv_psi_last_t;
  const uint32_t* gamma_psi_t;
  const uint32_t* betas;
  uint32_t thr, q_last;
  int L;
  int64_t N;
};

int rescale_run(const RescaleArgs& a, const uint32_t* X, int64_t xps, uint32_t* R, uint32_t* LL, uint32_t* tmp,
                int64_t polys, cudaStream_t st) {
  const int L1 = a.L - 1;
  const int64_t N = a.N, nv = N / 4;
  int rc;
  Epi twist;
  twist.op = EPI_MUL;
  twist.tab = a.inv_psi_last_t;
  twist.trow = a.m_zero;
  if ((rc = ntt_exec(a.ntt, true, LP{X + (int64_t)L1 * N, xps, 0}, COEF_NATURAL, LPo{LL, N, 0}, COEF_TRANSPOSED, polys,
                     1, a.m_last, twist, tmp, st)))
    return rc;
  {
    int64_t gb = (polys * nv + T - 1) / T;
    const unsigned g = (unsigned)(gb < 148 * 16 ? gb : 148 * 16);
    if (a.ntt->tc_fast)
      k_rescale_lift<true, true><<<g, T, 0, st>>>(LL, R, polys, L1, N, a.thr, a.q_last, a.gamma_psi_t, a.mods_q1);
    else if (plan_w32(a.ntt))
      k_rescale_lift<true, false><<<g, T, 0, st>>>(LL, R, polys, L1, N, a.thr, a.q_last, a.gamma_psi_t, a.mods_q1);
    else
      k_rescale_lift<false, false><<<g, T, 0, st>>>(LL, R, polys, L1, N, a.thr, a.q_last, a.gamma_psi_t, a.mods_q1);
  }
  count_launch();
  Epi comb;
  comb.op = EPI_COMBINE;
  comb.x = View{X, xps, 0, N, 1};
  comb.scal = a.betas;
  if ((rc = ntt_exec(a.ntt, false, LP{R, (int64_t)L1 * N, N}, COEF_TRANSPOSED, LPo{R, (int64_t)L1 * N, N},
                     COEF_NATURAL, polys, L1, a.m_q1, comb, tmp, st)))
    return rc;
  CROSS_CHECK_CUDA(cudaGetLastError());
  return CROSS_OK;
}
}  // namespace
}  // namespace cross

using namespace cross;

// ---------------------------------------------------------------------------
// HE-Mult
// ---------------------------------------------------------------------------

struct cross_hemul_plan_s {
  int r = 0, c = 0, L = 0, L1 = 0, K = 0, dnum = 0, alpha = 0, parts = 0;
  int64_t N = 0;
  cross_ntt_plan_s* ntt_qp = nullptr;
  cross_ntt_plan_s* ntt_p = nullptr;
  int p_off = 0;
  int down_layout = COEF_TRANSPOSED;   // coefficient order of the ModDown INTT / BConv / NTT
  std::vector<cross_bconv_plan_s*> ks_bconv;
  cross_bconv_plan_s* down = nullptr;
  std::vector<int> dstart, dlen;
  std::vector<std::vector<int>> comp;   // complement, indices in Q'+P
  std::vector<int> seq_host;            // 0, 1, ... (the ModDown twist rows)
  uint32_t thr = 0, q_last = 0;
  // device tables; _t = transposed coefficient order, _d = ModDown order
  uint32_t *inv_psi_last_t = nullptr, *gamma_psi_t = nullptr, *inv_psi_q_t = nullptr, *psi_qp_t = nullptr,
           *inv_psi_p_d = nullptr, *psi_q_d = nullptr, *betas = nullptr, *pinv = nullptr;
  ModC* mods_dle = nullptr;
  uint16_t *m_last = nullptr, *m_zero = nullptr, *seq = nullptr, *m_p_plan = nullptr, *m_q1_plan = nullptr;
  std::vector<uint16_t*> comp_plan, comp_dle;
  int16_t* ks_src = nullptr;
  uint32_t *evk_a = nullptr, *evk_b = nullptr;
};

namespace {

struct HemulBufs {
  uint32_t *X, *LL, *R, *D, *Cc, *KS, *KP, *F, *tmp, *O;
  std::vector<uint32_t*> E;
};

void hemul_layout(const cross_hemul_plan_s* P, int64_t B, int layout, Arena& a, HemulBufs& b) {
  const int64_t N = P->N;
  const int L = P->L, L1 = P->L1, K = P->K;
  b.X = layout == CROSS_LAYOUT_REFERENCE ? a.take<uint32_t>((size_t)B * 4 * L * N) : nullptr;
  b.LL = a.take<uint32_t>((size_t)B * 4 * N);
  b.R = a.take<uint32_t>((size_t)B * 4 * L1 * N);
  b.D = a.take<uint32_t>((size_t)B * 3 * L1 * N);
  b.Cc = a.take<uint32_t>((size_t)B * L1 * N);
  b.E.clear();
  for (int j = 0; j < P->parts; ++j) b.E.push_back(a.take<uint32_t>((size_t)B * (L1 + K - P->dlen[j]) * N));
  b.KS = a.take<uint32_t>((size_t)B * 2 * (L1 + K) * N);
  b.KP = a.take<uint32_t>((size_t)B * 2 * K * N);
  b.F = a.take<uint32_t>((size_t)B * 2 * L1 * N);
  b.O = layout == CROSS_LAYOUT_REFERENCE ? a.take<uint32_t>((size_t)B * 2 * L1 * N) : nullptr;
  int64_t tmpw = B * 4 * L1;
  for (int j = 0; j < P->parts; ++j) tmpw = std::max<int64_t>(tmpw, B * (L1 + K - P->dlen[j]));
  tmpw = std::max<int64_t>(tmpw, B * 2 * K);
  b.tmp = a.take<uint32_t>((size_t)std::max(ntt_tmp_words(P->ntt_qp, tmpw), ntt_tmp_words(P->ntt_p, tmpw)));
}

}  // namespace

extern "C" {

int cross_hemul_plan_destroy(cross_hemul_plan P) {
  if (!P) return CROSS_OK;
  for (void* p : {(void*)P->inv_psi_last_t, (void*)P->gamma_psi_t, (void*)P->inv_psi_q_t, (void*)P->psi_qp_t,
                  (void*)P->inv_psi_p_d, (void*)P->psi_q_d, (void*)P->betas, (void*)P->pinv, (void*)P->mods_dle,
                  (void*)P->m_last, (void*)P->m_zero, (void*)P->seq, (void*)P->m_p_plan, (void*)P->m_q1_plan,
                  (void*)P->ks_src, (void*)P->evk_a, (void*)P->evk_b})
    dfree(p);
  for (auto* p : P->comp_plan) dfree(p);
  for (auto* p : P->comp_dle) dfree(p);
  delete P;
  return CROSS_OK;
}

int cross_hemul_plan_create(const cross_hemul_desc* d, cross_hemul_plan* out) {
  CROSS_REQUIRE(d && out, "cross_hemul_plan_create: null argument");
  *out = nullptr;
  CROSS_REQUIRE(d->L >= 2 && d->K >= 1 && d->dnum >= 1 && d->r >= 1 && d->c >= 1,
                "cross_hemul_plan_create: need L >= 2, K >= 1, dnum >= 1");
  CROSS_REQUIRE(d->ntt_qp && d->ntt_p && d->ks_bconv && d->down_bconv && d->inv_psi_last && d->gamma_psi &&
                    d->betas && d->inv_psi_q && d->psi_qp && d->inv_psi_p && d->p_inv_mod_q,
                "cross_hemul_plan_create: null table or plan");
  CROSS_REQUIRE(d->ntt_qp->red == CROSS_REDUCTION_BARRETT && d->ntt_p->red == CROSS_REDUCTION_BARRETT &&
                    d->down_bconv->red == CROSS_REDUCTION_BARRETT,
                "cross_hemul_plan_create: HE-Mult runs on Barrett plans (hemul.py:58,69,98)");
  const int L = d->L, L1 = L - 1, K = d->K;
  const int64_t N = (int64_t)d->r * d->c;
  CROSS_REQUIRE(N % 4 == 0, "cross_hemul_plan_create: N=%lld must be a multiple of 4", (long long)N);
  CROSS_REQUIRE(d->ntt_qp->M == L + K && d->ntt_qp->r == d->r && d->ntt_qp->c == d->c,
                "cross_hemul_plan_create: ntt_qp must cover L+K=%d limbs with factorisation (%d, %d)", L + K, d->r, d->c);
  CROSS_REQUIRE(d->ntt_p->M >= d->ntt_p_limb_offset + K && (int64_t)d->ntt_p->r * d->ntt_p->c == N &&
                    d->ntt_p_limb_offset >= 0,
                "cross_hemul_plan_create: ntt_p does not cover the P limbs");
  auto* P = new cross_hemul_plan_s();
  P->r = d->r; P->c = d->c; P->L = L; P->L1 = L1; P->K = K; P->dnum = d->dnum; P->N = N;
  P->ntt_qp = d->ntt_qp; P->ntt_p = d->ntt_p; P->p_off = d->ntt_p_limb_offset;
  // The ModDown transforms keep transposed coefficients only when ntt_p has the
  // same (r, c) split as ntt_qp; otherwise natural order (factorisation-free).
  P->down_layout = (d->ntt_p->r == d->r && d->ntt_p->c == d->c) ? COEF_TRANSPOSED : COEF_NATURAL;
  P->alpha = (L1 + d->dnum - 1) / d->dnum;                     // ciphertext.py:354
  P->parts = (L1 + P->alpha - 1) / P->alpha;                   // ciphertext.py:356
  auto fail = [&](const char* msg, int q = -1) {
    set_error("cross_hemul_plan_create: %s (%d)", msg, q);
    cross_hemul_plan_destroy(P);
    return CROSS_ERR_INVALID_ARG;
  };
  if (P->parts > MAXPARTS) return fail("too many key-switch digits", P->parts);
  const auto& mq = d->ntt_qp->mods_host;
  std::vector<ModC> dle;
  for (int i = 0; i < L1; ++i) dle.push_back(mq[i]);
  for (int k = 0; k < K; ++k) dle.push_back(mq[L + k]);
  for (int k = 0; k < K; ++k)
    if (!same_q(d->ntt_p->mods_host[P->p_off + k], mq[L + k])) return fail("ntt_p moduli differ from P", k);
  const int LT = L1 + K;
  std::vector<int16_t> src((size_t)P->parts * LT, 0);
  for (int j = 0; j < P->parts; ++j) {
    const int s0 = j * P->alpha, len = std::min(P->alpha, L1 - s0);
    P->dstart.push_back(s0);
    P->dlen.push_back(len);
    std::vector<int> comp;
    for (int l = 0; l < LT; ++l)
      if (l < s0 || l >= s0 + len) comp.push_back(l);
    const cross_bconv_plan_s* bc = d->ks_bconv[j];
    if (!bc || bc->sq != len || bc->sp != (int)comp.size()) return fail("ks_bconv shape mismatch", j);
    for (int i = 0; i < len; ++i)
      if (!same_q(bc->src_host[i], dle[s0 + i])) return fail("ks_bconv source moduli", j);
    for (size_t i = 0; i < comp.size(); ++i)
      if (!same_q(bc->dst_host[i], dle[comp[i]])) return fail("ks_bconv target moduli", j);
    for (int l = 0; l < LT; ++l) src[(size_t)j * LT + l] = -1;
    for (size_t i = 0; i < comp.size(); ++i) src[(size_t)j * LT + comp[i]] = (int16_t)i;
    P->ks_bconv.push_back(d->ks_bconv[j]);
    P->comp.push_back(comp);
  }
  P->down = d->down_bconv;
  if (P->down->sq != K || P->down->sp != L1) return fail("down_bconv shape mismatch");
  for (int k = 0; k < K; ++k)
    if (!same_q(P->down->src_host[k], dle[L1 + k])) return fail("down_bconv source moduli", k);
  for (int i = 0; i < L1; ++i)
    if (!same_q(P->down->dst_host[i], dle[i])) return fail("down_bconv target moduli", i);
  P->q_last = (uint32_t)mq[L - 1].q;
  P->thr = (P->q_last + 1) / 2;                                 // ciphertext.py:260
  std::vector<uint16_t> seq(std::max<int>(LT, 4) + 1), last{(uint16_t)(L - 1)}, zero{0}, pp, q1;
  for (size_t i = 0; i < seq.size(); ++i) seq[i] = (uint16_t)i;
  P->seq_host.assign(seq.begin(), seq.end());
  for (int k = 0; k < K; ++k) pp.push_back((uint16_t)(P->p_off + k));
  for (int i = 0; i < L1; ++i) q1.push_back((uint16_t)i);
  const int R = d->r, C = d->c;
  int rc = CROSS_OK;
  auto upv = [&](uint32_t** dst, const std::vector<uint32_t>& v) { if (!rc) rc = upload_vec(dst, v); };
  upv(&P->inv_psi_last_t, to_transposed(d->inv_psi_last, 1, R, C));
  upv(&P->gamma_psi_t, to_transposed(d->gamma_psi, L1, R, C));
  upv(&P->inv_psi_q_t, to_transposed(d->inv_psi_q, L1, R, C));
  upv(&P->psi_qp_t, to_transposed(d->psi_qp, LT, R, C));
  if (P->down_layout == COEF_TRANSPOSED) {
    upv(&P->inv_psi_p_d, to_transposed(d->inv_psi_p, K, R, C));
    upv(&P->psi_q_d, to_transposed(d->psi_qp, L1, R, C));
  } else {
    upv(&P->inv_psi_p_d, std::vector<uint32_t>(d->inv_psi_p, d->inv_psi_p + (size_t)K * N));
    upv(&P->psi_q_d, std::vector<uint32_t>(d->psi_qp, d->psi_qp + (size_t)L1 * N));
  }
  if (!rc) rc = upload(&P->betas, d->betas, L1);
  if (!rc) rc = upload(&P->pinv, d->p_inv_mod_q, L1);
  if (!rc) rc = upload_vec(&P->mods_dle, dle);
  if (!rc) rc = upload_vec(&P->m_last, last);
  if (!rc) rc = upload_vec(&P->m_zero, zero);
  if (!rc) rc = upload_vec(&P->seq, seq);
  if (!rc) rc = upload_vec(&P->m_p_plan, pp);
  if (!rc) rc = upload_vec(&P->m_q1_plan, q1);
  if (!rc) rc = upload_vec(&P->ks_src, src);
  for (int j = 0; j < P->parts && !rc; ++j) {
    std::vector<uint16_t> cp, cd;
    for (int l : P->comp[j]) { cd.push_back((uint16_t)l); cp.push_back((uint16_t)(l < L1 ? l : l + 1)); }
    uint16_t *a = nullptr, *b = nullptr;
    rc = upload_vec(&a, cp);
    if (!rc) rc = upload_vec(&b, cd);
    P->comp_plan.push_back(a);
    P->comp_dle.push_back(b);
  }
  if (rc) {
    cross_hemul_plan_destroy(P);
    return rc;
  }
  *out = P;
  return CROSS_OK;
}

int cross_hemul_set_keys(cross_hemul_plan P, const uint32_t* evk_a, const uint32_t* evk_b, int key_limbs) {
  CROSS_REQUIRE(P && evk_a && evk_b, "cross_hemul_set_keys: null argument");
  const int L1 = P->L1, K = P->K, LT = L1 + K;
  CROSS_REQUIRE(key_limbs >= LT, "cross_hemul_set_keys: key has %d limbs, need >= %d", key_limbs, LT);
  const int64_t N = P->N;
  std::vector<uint32_t> a((size_t)P->parts * LT * N), b(a.size());
  // ciphertext.py:450-451: keep key limbs [0, L1) and the last K.
  for (int j = 0; j < P->parts; ++j)
    for (int l = 0; l < LT; ++l) {
      const int kl = l < L1 ? l : key_limbs - K + (l - L1);
      for (int64_t t = 0; t < N; ++t) {
        const size_t s = ((size_t)j * N + t) * key_limbs + kl;
        a[((size_t)j * LT + l) * N + t] = evk_a[s];
        b[((size_t)j * LT + l) * N + t] = evk_b[s];
      }
    }
  dfree(P->evk_a);
  dfree(P->evk_b);
  P->evk_a = P->evk_b = nullptr;
  int rc = upload_vec(&P->evk_a, a);
  if (!rc) rc = upload_vec(&P->evk_b, b);
  return rc;
}

size_t cross_hemul_workspace_size(cross_hemul_plan P, int64_t batch, int layout) {
  if (!P || batch < 0) return 0;
  Arena a(nullptr, 0);
  HemulBufs b;
  hemul_layout(P, batch, layout, a, b);
  return a.off;
}

int cross_hemul(cross_hemul_plan P, const uint32_t* in, uint32_t* out, int64_t B, int layout, void* ws,
                size_t ws_bytes, void* stream) {
  CROSS_REQUIRE(P && B >= 0 && (B == 0 || (in && out)), "cross_hemul: bad argument");
  CROSS_REQUIRE(P->evk_a && P->evk_b, "cross_hemul: keys not set (call cross_hemul_set_keys)");
  CROSS_REQUIRE(layout == CROSS_LAYOUT_REFERENCE || layout == CROSS_LAYOUT_LIMB_MAJOR, "cross_hemul: bad layout");
  CROSS_REQUIRE(layout == CROSS_LAYOUT_REFERENCE || (((uintptr_t)in | (uintptr_t)out) & 15) == 0,
                "cross_hemul: limb-major buffers must be 16-byte aligned");
  if (B == 0) return CROSS_OK;
  const size_t need = cross_hemul_workspace_size(P, B, layout);
  if (!ws || ws_bytes < need) {
    set_error("cross_hemul: workspace of %zu bytes required, %zu given", need, ws_bytes);
    return CROSS_ERR_WORKSPACE;
  }
  cudaStream_t st = (cudaStream_t)stream;
  const int64_t N = P->N;
  const int L = P->L, L1 = P->L1, K = P->K, LT = L1 + K;
  Arena a(ws, ws_bytes);
  HemulBufs b;
  hemul_layout(P, B, layout, a, b);
  int rc;
  const uint32_t* X = in;
  if (layout == CROSS_LAYOUT_REFERENCE) {
    if ((rc = transpose_u32(in, b.X, B * 4, N, L, st))) return rc;
    X = b.X;
  }
  const int64_t nv = N / 4;
  const dim3 blk(T);
  // 1. rescale (ciphertext.py:267-303)
  {
    RescaleArgs ra{P->ntt_qp, P->m_last, P->m_zero, P->m_q1_plan, P->mods_dle, P->inv_psi_last_t, P->gamma_psi_t,
                   P->betas, P->thr, P->q_last, L, N};
    if ((rc = rescale_run(ra, X, (int64_t)L * N, b.R, b.LL, b.tmp, B * 4, st))) return rc;
  }
  // 2. tensor product (ciphertext.py:309-324)
  const bool w32 = plan_w32(P->ntt_qp);
  if (w32)
    k_tensor_lm<true><<<dim3(gx_for(nv), gy_for(B * L1)), blk, 0, st>>>(b.R, b.D, B, L1, N, P->mods_dle);
  else
    k_tensor_lm<false><<<dim3(gx_for(nv), gy_for(B * L1)), blk, 0, st>>>(b.R, b.D, B, L1, N, P->mods_dle);
  count_launch();
  // 3. key switch on d2 (ciphertext.py:455-519): INTT x psi^-i (fused, transposed
  // coefficients) -> per digit BConv x psi^i (fused) -> NTT -> inner product
  const uint32_t* D2 = b.D + 2 * (int64_t)L1 * N;
  const int64_t Dps = 3 * (int64_t)L1 * N;
  Epi tw;
  tw.op = EPI_MUL;
  tw.tab = P->inv_psi_q_t;
  tw.trow = P->seq;
  if ((rc = ntt_exec(P->ntt_qp, true, LP{D2, Dps, N}, COEF_NATURAL, LPo{b.Cc, (int64_t)L1 * N, N}, COEF_TRANSPOSED, B,
                     L1, P->m_q1_plan, tw, b.tmp, st)))
    return rc;
  PartPtrs pp{};
  for (int j = 0; j < P->parts; ++j) {
    const int ns = LT - P->dlen[j];
    const int64_t eps = (int64_t)ns * N;
    if ((rc = bconv_run(P->ks_bconv[j], true, b.Cc + (int64_t)P->dstart[j] * N, (int64_t)L1 * N, N, 1, b.E[j], eps,
                        N, 1, B, N, st, P->psi_qp_t, P->comp_dle[j], P->comp[j].data())))
      return rc;
    if ((rc = ntt_exec(P->ntt_qp, false, LP{b.E[j], eps, N}, COEF_TRANSPOSED, LPo{b.E[j], eps, N}, COEF_NATURAL, B, ns,
                       P->comp_plan[j], Epi{}, b.tmp, st)))
      return rc;
    pp.e[j] = b.E[j];
    pp.ps[j] = eps;
  }
  if ((rc = ks_inner(w32, LP{D2, Dps, N}, pp, P->parts, P->ks_src, LT, N, B, P->evk_a, P->evk_b, b.KS, P->mods_dle,
                     st)))
    return rc;
  // 4. ModDown (hemul.py:175-215): INTT of the P limbs of both elements x psi^-i
  // -> BConv P -> Q' x psi^i -> NTT whose last stage applies the subtraction, the
  // P^-1 scaling and the add of (d0, d1).  Element e of ciphertext b is e' = 2b + e.
  const int64_t KSes = (int64_t)LT * N;
  tw.tab = P->inv_psi_p_d;
  if ((rc = ntt_exec(P->ntt_p, true, LP{b.KS + (int64_t)L1 * N, KSes, N}, COEF_NATURAL, LPo{b.KP, (int64_t)K * N, N},
                     P->down_layout, B * 2, K, P->m_p_plan, tw, b.tmp, st)))
    return rc;
  if ((rc = bconv_run(P->down, true, b.KP, (int64_t)K * N, N, 1, b.F, (int64_t)L1 * N, N, 1, B * 2, N, st, P->psi_q_d,
                      P->seq, P->seq_host.data())))
    return rc;
  Epi md;
  md.op = EPI_MODDOWN;
  md.x = View{b.KS, KSes, 0, N, 1};
  md.scal = P->pinv;
  md.base = View{b.D, Dps, (int64_t)L1 * N, N, 2};
  md.base_mask = 3u;
  uint32_t* O = layout == CROSS_LAYOUT_REFERENCE ? b.O : out;
  if ((rc = ntt_exec(P->ntt_qp, false, LP{b.F, (int64_t)L1 * N, N}, P->down_layout, LPo{O, (int64_t)L1 * N, N},
                     COEF_NATURAL, B * 2, L1, P->m_q1_plan, md, b.tmp, st)))
    return rc;
  CROSS_CHECK_CUDA(cudaGetLastError());
  if (layout == CROSS_LAYOUT_REFERENCE) return transpose_u32(b.O, out, B * 2, L1, N, st);
  return CROSS_OK;
}

}  // extern "C"

// ---------------------------------------------------------------------------
// HE-Rotate
// ---------------------------------------------------------------------------

struct cross_herot_plan_s {
  int L = 0, K = 0, dnum = 0, alpha = 0, parts = 0;
  int64_t N = 0;
  cross_ntt_plan_s* ntt = nullptr;
  std::vector<cross_bconv_plan_s*> ks_bconv;
  cross_bconv_plan_s* down = nullptr;
  std::vector<int> dstart, dlen;
  // coefficient-order tables, transposed for the (r, c) split of the plan
  uint32_t *inv_psi_q_t = nullptr, *psi_qp_t = nullptr, *inv_psi_p_t = nullptr, *pinv = nullptr;
  uint16_t *seq = nullptr, *m_p = nullptr;
  std::vector<uint16_t*> comp;
  std::vector<std::vector<int>> comp_host;   // the same complements on the host
  std::vector<int> seq_host;
  int16_t* ks_src = nullptr;
  uint32_t *evk_a = nullptr, *evk_b = nullptr;
  int32_t* coef_map = nullptr;
};

namespace {

struct HerotBufs {
  uint32_t *X, *Cq, *KS, *KP, *F, *Rz, *tmp, *Tr;
  std::vector<uint32_t*> E;
};

void herot_layout(const cross_herot_plan_s* P, int64_t B, int layout, Arena& a, HerotBufs& b) {
  const int64_t N = P->N;
  const int L = P->L, K = P->K;
  b.X = layout == CROSS_LAYOUT_REFERENCE ? a.take<uint32_t>((size_t)B * 2 * L * N) : nullptr;
  b.Cq = a.take<uint32_t>((size_t)B * L * N);
  b.E.clear();
  for (int j = 0; j < P->parts; ++j) b.E.push_back(a.take<uint32_t>((size_t)B * (L + K - P->dlen[j]) * N));
  b.KS = a.take<uint32_t>((size_t)B * 2 * (L + K) * N);
  b.KP = a.take<uint32_t>((size_t)B * 2 * K * N);
  b.F = a.take<uint32_t>((size_t)B * 2 * L * N);
  b.Rz = a.take<uint32_t>((size_t)B * 2 * L * N);
  b.Tr = layout == CROSS_LAYOUT_REFERENCE ? a.take<uint32_t>((size_t)B * 2 * L * N) : nullptr;
  int64_t tmpw = B * std::max(L, 2 * K);
  for (int j = 0; j < P->parts; ++j) tmpw = std::max<int64_t>(tmpw, B * (L + K - P->dlen[j]));
  tmpw = std::max<int64_t>(tmpw, B * 2 * L);
  b.tmp = a.take<uint32_t>((size_t)ntt_tmp_words(P->ntt, tmpw));
}

}  // namespace

extern "C" {

int cross_herot_plan_destroy(cross_herot_plan P) {
  if (!P) return CROSS_OK;
  for (void* p : {(void*)P->inv_psi_q_t, (void*)P->psi_qp_t, (void*)P->inv_psi_p_t, (void*)P->pinv, (void*)P->seq,
                  (void*)P->m_p, (void*)P->ks_src, (void*)P->evk_a, (void*)P->evk_b, (void*)P->coef_map})
    dfree(p);
  for (auto* p : P->comp) dfree(p);
  delete P;
  return CROSS_OK;
}

int cross_herot_plan_create(const cross_herot_desc* d, cross_herot_plan* out) {
  CROSS_REQUIRE(d && out, "cross_herot_plan_create: null argument");
  *out = nullptr;
  CROSS_REQUIRE(d->L >= 1 && d->K >= 1 && d->dnum >= 1 && d->ntt_qp && d->ks_bconv && d->down_bconv &&
                    d->inv_psi_q && d->psi_qp && d->inv_psi_p && d->p_inv_mod_q,
                "cross_herot_plan_create: bad descriptor");
  CROSS_REQUIRE(d->ntt_qp->red == CROSS_REDUCTION_BARRETT && d->down_bconv->red == CROSS_REDUCTION_BARRETT,
                "cross_herot_plan_create: HE-Rotate runs on Barrett plans (herot.py:64, 161-175)");
  const int L = d->L, K = d->K, LT = L + K;
  const int64_t N = (int64_t)d->r * d->c;
  CROSS_REQUIRE(N % 4 == 0 && d->ntt_qp->M == LT && (int64_t)d->ntt_qp->r * d->ntt_qp->c == N,
                "cross_herot_plan_create: ntt_qp must cover L+K limbs of N");
  auto* P = new cross_herot_plan_s();
  P->L = L; P->K = K; P->dnum = d->dnum; P->N = N; P->ntt = d->ntt_qp;
  P->alpha = (L + d->dnum - 1) / d->dnum;                       // herot.py:73
  P->parts = (L + P->alpha - 1) / P->alpha;                     // herot.py:119
  auto fail = [&](const char* msg, int q = -1) {
    set_error("cross_herot_plan_create: %s (%d)", msg, q);
    cross_herot_plan_destroy(P);
    return CROSS_ERR_INVALID_ARG;
  };
  // herot.py:212 loops over dnum digits; the reference fails with an
  // IndexError when fewer than dnum digits exist.
  if (P->parts < d->dnum) return fail("dnum exceeds the number of digits ceil(L/alpha)", P->parts);
  if (P->parts > MAXPARTS) return fail("too many key-switch digits", P->parts);
  const auto& mq = d->ntt_qp->mods_host;
  std::vector<int16_t> src((size_t)d->dnum * LT, -1);
  for (int j = 0; j < d->dnum; ++j) {
    const int s0 = j * P->alpha, len = std::min(P->alpha, L - s0);
    P->dstart.push_back(s0);
    P->dlen.push_back(len);
    std::vector<int> comp;
    for (int l = 0; l < LT; ++l)
      if (l < s0 || l >= s0 + len) comp.push_back(l);
    const cross_bconv_plan_s* bc = d->ks_bconv[j];
    if (!bc || bc->sq != len || bc->sp != (int)comp.size()) return fail("ks_bconv shape mismatch", j);
    for (int i = 0; i < len; ++i)
      if (!same_q(bc->src_host[i], mq[s0 + i])) return fail("ks_bconv source moduli", j);
    for (size_t i = 0; i < comp.size(); ++i)
      if (!same_q(bc->dst_host[i], mq[comp[i]])) return fail("ks_bconv target moduli", j);
    for (size_t i = 0; i < comp.size(); ++i) src[(size_t)j * LT + comp[i]] = (int16_t)i;
    P->ks_bconv.push_back(d->ks_bconv[j]);
    P->comp_host.push_back(comp);
    std::vector<uint16_t> cu(comp.begin(), comp.end());
    uint16_t* dp = nullptr;
    if (upload_vec(&dp, cu)) return fail("upload");
    P->comp.push_back(dp);
  }
  P->parts = d->dnum;
  P->down = d->down_bconv;
  if (P->down->sq != K || P->down->sp != L) return fail("down_bconv shape mismatch");
  std::vector<uint16_t> seq(LT + 1), mp;
  for (size_t i = 0; i < seq.size(); ++i) seq[i] = (uint16_t)i;
  P->seq_host.assign(seq.begin(), seq.end());
  for (int k = 0; k < K; ++k) mp.push_back((uint16_t)(L + k));
  int rc = CROSS_OK;
  const int R = d->ntt_qp->r, C = d->ntt_qp->c;
  auto upv = [&](uint32_t** dst, const std::vector<uint32_t>& v) { if (!rc) rc = upload_vec(dst, v); };
  upv(&P->inv_psi_q_t, to_transposed(d->inv_psi_q, L, R, C));
  upv(&P->psi_qp_t, to_transposed(d->psi_qp, LT, R, C));
  upv(&P->inv_psi_p_t, to_transposed(d->inv_psi_p, K, R, C));
  if (!rc) rc = upload(&P->pinv, d->p_inv_mod_q, L);
  if (!rc) rc = upload_vec(&P->seq, seq);
  if (!rc) rc = upload_vec(&P->m_p, mp);
  if (!rc) rc = upload_vec(&P->ks_src, src);
  if (rc) {
    cross_herot_plan_destroy(P);
    return rc;
  }
  *out = P;
  return CROSS_OK;
}

int cross_herot_set_keys(cross_herot_plan P, const uint32_t* evk_a, const uint32_t* evk_b, const int32_t* coef_map) {
  CROSS_REQUIRE(P && evk_a && evk_b && coef_map, "cross_herot_set_keys: null argument");
  const int LT = P->L + P->K;
  const int64_t N = P->N;
  std::vector<uint32_t> a((size_t)P->parts * LT * N), b(a.size());
  for (int j = 0; j < P->parts; ++j)
    for (int l = 0; l < LT; ++l)
      for (int64_t t = 0; t < N; ++t) {
        const size_t s = ((size_t)j * N + t) * LT + l;
        a[((size_t)j * LT + l) * N + t] = evk_a[s];
        b[((size_t)j * LT + l) * N + t] = evk_b[s];
      }
  dfree(P->evk_a);
  dfree(P->evk_b);
  dfree(P->coef_map);
  P->evk_a = P->evk_b = nullptr;
  P->coef_map = nullptr;
  int rc = upload_vec(&P->evk_a, a);
  if (!rc) rc = upload_vec(&P->evk_b, b);
  if (!rc) rc = upload(&P->coef_map, coef_map, (size_t)N);
  return rc;
}

size_t cross_herot_workspace_size(cross_herot_plan P, int64_t batch, int layout) {
  if (!P || batch < 0) return 0;
  Arena a(nullptr, 0);
  HerotBufs b;
  herot_layout(P, batch, layout, a, b);
  return a.off;
}

int cross_herot(cross_herot_plan P, const uint32_t* in, uint32_t* out, int64_t B, int layout, void* ws,
                size_t ws_bytes, void* stream) {
  CROSS_REQUIRE(P && B >= 0 && (B == 0 || (in && out)), "cross_herot: bad argument");
  CROSS_REQUIRE(P->evk_a && P->evk_b && P->coef_map, "cross_herot: keys not set (call cross_herot_set_keys)");
  CROSS_REQUIRE(layout == CROSS_LAYOUT_REFERENCE || layout == CROSS_LAYOUT_LIMB_MAJOR, "cross_herot: bad layout");
  CROSS_REQUIRE(layout == CROSS_LAYOUT_REFERENCE || (((uintptr_t)in | (uintptr_t)out) & 15) == 0,
                "cross_herot: limb-major buffers must be 16-byte aligned");
  if (B == 0) return CROSS_OK;
  const size_t need = cross_herot_workspace_size(P, B, layout);
  if (!ws || ws_bytes < need) {
    set_error("cross_herot: workspace of %zu bytes required, %zu given", need, ws_bytes);
    return CROSS_ERR_WORKSPACE;
  }
  cudaStream_t st = (cudaStream_t)stream;
  const int64_t N = P->N;
  const int L = P->L, K = P->K, LT = L + K;
  Arena a(ws, ws_bytes);
  HerotBufs b;
  herot_layout(P, B, layout, a, b);
  int rc;
  const uint32_t* X = in;
  if (layout == CROSS_LAYOUT_REFERENCE) {
    if ((rc = transpose_u32(in, b.X, B * 2, N, L, st))) return rc;
    X = b.X;
  }
  const dim3 blk(T);
  const int64_t Xps = 2 * (int64_t)L * N;
  const uint32_t* X1 = X + (int64_t)L * N;   // in_tower = element 1 (herot.py:201)
  // 1. key switch of element 1 (herot.py:203-247): INTT x psi^-i (fused,
  // transposed coefficients) -> per digit BConv x psi^i -> NTT -> inner product
  Epi tw;
  tw.op = EPI_MUL;
  tw.tab = P->inv_psi_q_t;
  tw.trow = P->seq;
  if ((rc = ntt_exec(P->ntt, true, LP{X1, Xps, N}, COEF_NATURAL, LPo{b.Cq, (int64_t)L * N, N}, COEF_TRANSPOSED, B, L,
                     P->seq, tw, b.tmp, st)))
    return rc;
  PartPtrs pp{};
  for (int j = 0; j < P->parts; ++j) {
    const int ns = LT - P->dlen[j];
    const int64_t eps = (int64_t)ns * N;
    if ((rc = bconv_run(P->ks_bconv[j], true, b.Cq + (int64_t)P->dstart[j] * N, (int64_t)L * N, N, 1, b.E[j], eps, N,
                        1, B, N, st, P->psi_qp_t, P->comp[j], P->comp_host[j].data())))
      return rc;
    if ((rc = ntt_exec(P->ntt, false, LP{b.E[j], eps, N}, COEF_TRANSPOSED, LPo{b.E[j], eps, N}, COEF_NATURAL, B, ns,
                       P->comp[j], Epi{}, b.tmp, st)))
      return rc;
    pp.e[j] = b.E[j];
    pp.ps[j] = eps;
  }
  if ((rc = ks_inner(plan_w32(P->ntt), LP{X1, Xps, N}, pp, P->parts, P->ks_src, LT, N, B, P->evk_a, P->evk_b, b.KS,
                     P->ntt->mods, st)))
    return rc;
  // 2. ModDown of both elements (herot.py:255-289) and c0 += ModDown_0
  // (herot.py:292-296), the tail fused into the last NTT stage.
  const int64_t KSes = (int64_t)LT * N;
  tw.tab = P->inv_psi_p_t;
  if ((rc = ntt_exec(P->ntt, true, LP{b.KS + (int64_t)L * N, KSes, N}, COEF_NATURAL, LPo{b.KP, (int64_t)K * N, N},
                     COEF_TRANSPOSED, B * 2, K, P->m_p, tw, b.tmp, st)))
    return rc;
  if ((rc = bconv_run(P->down, true, b.KP, (int64_t)K * N, N, 1, b.F, (int64_t)L * N, N, 1, B * 2, N, st, P->psi_qp_t,
                      P->seq, P->seq_host.data())))
    return rc;
  Epi md;
  md.op = EPI_MODDOWN;
  md.x = View{b.KS, KSes, 0, N, 1};
  md.scal = P->pinv;
  md.base = View{X, Xps, (int64_t)L * N, N, 2};
  md.base_mask = 1u;
  if ((rc = ntt_exec(P->ntt, false, LP{b.F, (int64_t)L * N, N}, COEF_TRANSPOSED, LPo{b.Rz, (int64_t)L * N, N},
                     COEF_NATURAL, B * 2, L, P->seq, md, b.tmp, st)))
    return rc;
  CROSS_CHECK_CUDA(cudaGetLastError());
  // 4. automorphism (herot.py:300)
  if (layout == CROSS_LAYOUT_REFERENCE) {
    if ((rc = transpose_u32(b.Rz, b.Tr, B * 2, L, N, st))) return rc;
    return cross_automorphism(b.Tr, P->coef_map, out, B * 2, N, L, st);
  }
  const int64_t rows = B * 2 * L;
  k_gather_lm<<<dim3((unsigned)((N + T - 1) / T > 64 ? 64 : (N + T - 1) / T), gy_for(rows)), blk, 0, st>>>(
      b.Rz, P->coef_map, out, rows, N); count_launch();
  CROSS_CHECK_CUDA(cudaGetLastError());
  return CROSS_OK;
}

}  // extern "C"

// ---------------------------------------------------------------------------
// Standalone rescale
// ---------------------------------------------------------------------------

struct cross_rescale_plan_s {
  int L = 0;
  int64_t N = 0;
  cross_ntt_plan_s* ntt = nullptr;
  uint32_t *inv_psi_last_t = nullptr, *gamma_psi_t = nullptr, *betas = nullptr;
  uint16_t *m_last = nullptr, *m_zero = nullptr, *m_q1 = nullptr;
  uint32_t thr = 0, q_last = 0;
};

namespace {
struct RescaleBufs {
  uint32_t *X, *R, *LL, *tmp;
};
void rescale_layout(const cross_rescale_plan_s* P, int64_t polys, int layout, Arena& a, RescaleBufs& b) {
  const int64_t N = P->N;
  b.X = layout == CROSS_LAYOUT_REFERENCE ? a.take<uint32_t>((size_t)polys * P->L * N) : nullptr;
  b.R = layout == CROSS_LAYOUT_REFERENCE ? a.take<uint32_t>((size_t)polys * (P->L - 1) * N) : nullptr;
  b.LL = a.take<uint32_t>((size_t)polys * N);
  b.tmp = a.take<uint32_t>((size_t)ntt_tmp_words(P->ntt, polys * (P->L - 1)));
}
}  // namespace

extern "C" {

int cross_rescale_plan_destroy(cross_rescale_plan P) {
  if (!P) return CROSS_OK;
  for (void* p : {(void*)P->inv_psi_last_t, (void*)P->gamma_psi_t, (void*)P->betas, (void*)P->m_last,
                  (void*)P->m_zero, (void*)P->m_q1})
    dfree(p);
  delete P;
  return CROSS_OK;
}

int cross_rescale_plan_create(const cross_rescale_desc* d, cross_rescale_plan* out) {
  CROSS_REQUIRE(d && out && d->ntt_q && d->inv_psi_last && d->gamma_psi && d->betas && d->L >= 2,
                "cross_rescale_plan_create: bad descriptor");
  CROSS_REQUIRE(d->ntt_q->red == CROSS_REDUCTION_BARRETT,
                "cross_rescale_plan_create: rescale runs on a Barrett plan (ciphertext.py:251)");
  *out = nullptr;
  const int64_t N = (int64_t)d->r * d->c;
  CROSS_REQUIRE(N % 4 == 0 && (int64_t)d->ntt_q->r * d->ntt_q->c == N && d->ntt_q->M >= d->L,
                "cross_rescale_plan_create: ntt_q must cover the L moduli with N = r*c (N %% 4 == 0)");
  auto* P = new cross_rescale_plan_s();
  P->L = d->L;
  P->N = N;
  P->ntt = d->ntt_q;
  P->q_last = (uint32_t)d->ntt_q->mods_host[d->L - 1].q;
  P->thr = (P->q_last + 1) / 2;
  std::vector<uint16_t> last{(uint16_t)(d->L - 1)}, zero{0}, q1;
  for (int i = 0; i < d->L - 1; ++i) q1.push_back((uint16_t)i);
  int rc = upload_vec(&P->inv_psi_last_t, to_transposed(d->inv_psi_last, 1, d->ntt_q->r, d->ntt_q->c));
  if (!rc) rc = upload_vec(&P->gamma_psi_t, to_transposed(d->gamma_psi, d->L - 1, d->ntt_q->r, d->ntt_q->c));
  if (!rc) rc = upload(&P->betas, d->betas, (size_t)(d->L - 1));
  if (!rc) rc = upload_vec(&P->m_last, last);
  if (!rc) rc = upload_vec(&P->m_zero, zero);
  if (!rc) rc = upload_vec(&P->m_q1, q1);
  if (rc) {
    cross_rescale_plan_destroy(P);
    return rc;
  }
  *out = P;
  return CROSS_OK;
}

size_t cross_rescale_workspace_size(cross_rescale_plan P, int64_t polys, int layout) {
  if (!P || polys < 0) return 0;
  Arena a(nullptr, 0);
  RescaleBufs b;
  rescale_layout(P, polys, layout, a, b);
  return a.off;
}

int cross_rescale(cross_rescale_plan P, const uint32_t* in, uint32_t* out, int64_t polys, int layout, void* ws,
                  size_t ws_bytes, void* stream) {
  CROSS_REQUIRE(P && polys >= 0 && (polys == 0 || (in && out)), "cross_rescale: bad argument");
  CROSS_REQUIRE(layout == CROSS_LAYOUT_REFERENCE || layout == CROSS_LAYOUT_LIMB_MAJOR, "cross_rescale: bad layout");
  if (polys == 0) return CROSS_OK;
  const size_t need = cross_rescale_workspace_size(P, polys, layout);
  if (!ws || ws_bytes < need) {
    set_error("cross_rescale: workspace of %zu bytes required, %zu given", need, ws_bytes);
    return CROSS_ERR_WORKSPACE;
  }
  CROSS_REQUIRE(layout == CROSS_LAYOUT_REFERENCE || in != out, "cross_rescale: limb-major in and out must differ");
  CROSS_REQUIRE(layout == CROSS_LAYOUT_REFERENCE || (((uintptr_t)in | (uintptr_t)out) & 15) == 0,
                "cross_rescale: limb-major buffers must be 16-byte aligned");
  cudaStream_t st = (cudaStream_t)stream;
  const int64_t N = P->N;
  const int L = P->L;
  Arena a(ws, ws_bytes);
  RescaleBufs b;
  rescale_layout(P, polys, layout, a, b);
  // Barrett constants of Q' are the first L-1 entries of the plan's table.
  RescaleArgs ra{P->ntt, P->m_last, P->m_zero, P->m_q1, P->ntt->mods, P->inv_psi_last_t, P->gamma_psi_t, P->betas,
                 P->thr, P->q_last, L, N};
  int rc;
  if (layout == CROSS_LAYOUT_LIMB_MAJOR) return rescale_run(ra, in, (int64_t)L * N, out, b.LL, b.tmp, polys, st);
  if ((rc = transpose_u32(in, b.X, polys, N, L, st))) return rc;
  if ((rc = rescale_run(ra, b.X, (int64_t)L * N, b.R, b.LL, b.tmp, polys, st))) return rc;
  return transpose_u32(b.R, out, polys, L - 1, N, st);
}

}  // extern "C"

// ---------------------------------------------------------------------------
// HE-Mult sharded by RNS limb (one rank per GPU).  Rank g owns the Q' limbs
// [q0, q1) and the P limbs [p0, p1) of every ciphertext and computes exactly
// the per-limb operations of cross_hemul for them, so its output limbs are
// bit-identical to the one-GPU result.  The key switch needs two exchanges,
// done by the caller between the phases (an all-gather over the ranks):
//   1. ModUp: every digit's limbs of INTT(d2) psi^-i in coefficient form
//      (cc, limb-outer: Q' limb l at index l);
//   2. ModDown: the P limbs of INTT(KS) psi^-i of both elements (kp, limb-outer:
//      P limb k at index k).
// Everything else -- rescale, tensor product, the ModUp basis conversions into
// the rank's own limbs, the NTTs, the inner product and the ModDown tail -- is
// limb-local.
// ---------------------------------------------------------------------------

struct cross_hemul_shard_s {
  const cross_hemul_plan_s* P = nullptr;
  int q0 = 0, q1 = 0, p0 = 0, p1 = 0, nq = 0, np = 0, lt = 0;
  std::vector<cross_bconv_plan_s*> ks;          // per digit (nullptr when the rank has no target)
  std::vector<int> ns;                          // targets per digit
  std::vector<std::vector<int>> tgt_dle;        // targets per digit, indices in Q' + P
  cross_bconv_plan_s* down = nullptr;
  ModC* mods_own = nullptr;                     // [lt] own Q' then own P
  uint16_t *m_q = nullptr, *m_p = nullptr, *rows_p = nullptr;
  std::vector<uint16_t*> tgt_plan, tgt_rows;
  std::vector<int> q_rows_host;                 // q0 .. q1 - 1
  int16_t* src = nullptr;                       // [parts][lt]
  uint32_t *evk_a = nullptr, *evk_b = nullptr;  // [parts][lt][N]
};

namespace {

struct ShardBufs {
  uint32_t *LL, *R, *D, *KS, *F, *tmp;
  std::vector<uint32_t*> E;
};

void shard_layout(const cross_hemul_shard_s* S, int64_t B, Arena& a, ShardBufs& b) {
  const int64_t N = S->P->N;
  b.LL = a.take<uint32_t>((size_t)B * 4 * N);
  b.R = a.take<uint32_t>((size_t)B * 4 * S->nq * N);
  b.D = a.take<uint32_t>((size_t)B * 3 * S->nq * N);
  b.E.clear();
  int64_t tw = B * 4 * std::max(S->nq, 1);
  for (size_t j = 0; j < S->ns.size(); ++j) {
    b.E.push_back(a.take<uint32_t>((size_t)B * S->ns[j] * N));
    tw = std::max<int64_t>(tw, B * S->ns[j]);
  }
  b.KS = a.take<uint32_t>((size_t)B * 2 * S->lt * N);
  b.F = a.take<uint32_t>((size_t)B * 2 * S->nq * N);
  tw = std::max<int64_t>(tw, B * 2 * std::max(S->nq, S->np));
  b.tmp = a.take<uint32_t>((size_t)std::max(ntt_tmp_words(S->P->ntt_qp, tw), ntt_tmp_words(S->P->ntt_p, tw)));
}

int shard_ws_check(const cross_hemul_shard_s* S, int64_t B, void* ws, size_t bytes, ShardBufs& b, const char* who) {
  Arena q(nullptr, 0);
  shard_layout(S, B, q, b);
  if (!ws || bytes < q.off) {
    set_error("%s: workspace of %zu bytes required, %zu given", who, q.off, bytes);
    return CROSS_ERR_WORKSPACE;
  }
  Arena a(ws, bytes);
  shard_layout(S, B, a, b);
  return CROSS_OK;
}

}  // namespace

extern "C" {

int cross_hemul_shard_destroy(cross_hemul_shard S) {
  if (!S) return CROSS_OK;
  for (void* p : {(void*)S->mods_own, (void*)S->m_q, (void*)S->m_p, (void*)S->rows_p, (void*)S->src,
                  (void*)S->evk_a, (void*)S->evk_b})
    dfree(p);
  for (auto* p : S->tgt_plan) dfree(p);
  for (auto* p : S->tgt_rows) dfree(p);
  delete S;
  return CROSS_OK;
}

int cross_hemul_shard_create(const cross_hemul_shard_desc* d, cross_hemul_shard* out) {
  CROSS_REQUIRE(d && out && d->plan, "cross_hemul_shard_create: null argument");
  *out = nullptr;
  const cross_hemul_plan_s* P = d->plan;
  CROSS_REQUIRE(P->evk_a && P->evk_b, "cross_hemul_shard_create: the plan's keys are not set");
  CROSS_REQUIRE(0 <= d->q_begin && d->q_begin <= d->q_end && d->q_end <= P->L1 && 0 <= d->p_begin &&
                    d->p_begin <= d->p_end && d->p_end <= P->K,
                "cross_hemul_shard_create: limb ranges [%d, %d) of Q' (%d) and [%d, %d) of P (%d) out of range",
                d->q_begin, d->q_end, P->L1, d->p_begin, d->p_end, P->K);
  auto* S = new cross_hemul_shard_s();
  S->P = P;
  S->q0 = d->q_begin; S->q1 = d->q_end; S->p0 = d->p_begin; S->p1 = d->p_end;
  S->nq = S->q1 - S->q0; S->np = S->p1 - S->p0; S->lt = S->nq + S->np;
  const int L1 = P->L1, LT = L1 + P->K;
  auto fail = [&](const char* msg, int j) {
    set_error("cross_hemul_shard_create: %s (%d)", msg, j);
    cross_hemul_shard_destroy(S);
    return CROSS_ERR_INVALID_ARG;
  };
  // own limbs in Q' + P order: Q' [q0, q1) then P [p0, p1) (dle indices)
  std::vector<int> own;
  for (int l = S->q0; l < S->q1; ++l) own.push_back(l);
  for (int k = S->p0; k < S->p1; ++k) own.push_back(L1 + k);
  const auto& mq = P->ntt_qp->mods_host;
  auto dle_mod = [&](int l) { return l < L1 ? mq[l] : mq[P->L + (l - L1)]; };
  std::vector<int16_t> src((size_t)P->parts * std::max(S->lt, 1), -1);
  for (int j = 0; j < P->parts; ++j) {
    std::vector<int> tg;
    for (int l : own)
      if (l < P->dstart[j] || l >= P->dstart[j] + P->dlen[j]) tg.push_back(l);
    S->tgt_dle.push_back(tg);
    S->ns.push_back((int)tg.size());
    for (size_t i = 0; i < tg.size(); ++i)
      for (int s = 0; s < S->lt; ++s)
        if (own[s] == tg[i]) src[(size_t)j * S->lt + s] = (int16_t)i;
    cross_bconv_plan_s* bc = d->ks_bconv ? d->ks_bconv[j] : nullptr;
    if (!tg.empty()) {
      if (!bc || bc->red != CROSS_REDUCTION_BARRETT || bc->sq != P->dlen[j] || bc->sp != (int)tg.size())
        return fail("ks_bconv shape mismatch", j);
      for (int i = 0; i < bc->sq; ++i)
        if (!same_q(bc->src_host[i], dle_mod(P->dstart[j] + i))) return fail("ks_bconv source moduli", j);
      for (size_t i = 0; i < tg.size(); ++i)
        if (!same_q(bc->dst_host[i], dle_mod(tg[i]))) return fail("ks_bconv target moduli", j);
    }
    S->ks.push_back(tg.empty() ? nullptr : bc);
  }
  if (S->nq > 0) {
    S->down = d->down_bconv;
    if (!S->down || S->down->red != CROSS_REDUCTION_BARRETT || S->down->sq != P->K || S->down->sp != S->nq)
      return fail("down_bconv shape mismatch", S->nq);
    for (int k = 0; k < P->K; ++k)
      if (!same_q(S->down->src_host[k], mq[P->L + k])) return fail("down_bconv source moduli", k);
    for (int i = 0; i < S->nq; ++i)
      if (!same_q(S->down->dst_host[i], mq[S->q0 + i])) return fail("down_bconv target moduli", i);
  }
  std::vector<ModC> mo;
  for (int l : own) mo.push_back(dle_mod(l));
  std::vector<uint16_t> mqv, mpv, rpv;
  for (int l = S->q0; l < S->q1; ++l) { mqv.push_back((uint16_t)l); S->q_rows_host.push_back(l); }
  for (int k = S->p0; k < S->p1; ++k) { mpv.push_back((uint16_t)(P->p_off + k)); rpv.push_back((uint16_t)k); }
  int rc = CROSS_OK;
  if (!mo.empty()) rc = upload_vec(&S->mods_own, mo);
  if (!rc && !mqv.empty()) rc = upload_vec(&S->m_q, mqv);
  if (!rc && !mpv.empty()) rc = upload_vec(&S->m_p, mpv);
  if (!rc && !rpv.empty()) rc = upload_vec(&S->rows_p, rpv);
  if (!rc) rc = upload_vec(&S->src, src);
  for (int j = 0; j < P->parts && !rc; ++j) {
    std::vector<uint16_t> tp, tr;
    for (int l : S->tgt_dle[j]) { tr.push_back((uint16_t)l); tp.push_back((uint16_t)(l < L1 ? l : l + 1)); }
    uint16_t *a = nullptr, *b = nullptr;
    if (!tp.empty()) {
      rc = upload_vec(&a, tp);
      if (!rc) rc = upload_vec(&b, tr);
    }
    S->tgt_plan.push_back(a);
    S->tgt_rows.push_back(b);
  }
  // the owned rows of the evaluation keys, [parts][lt][N]
  const int64_t N = P->N;
  if (!rc && S->lt > 0) {
    const size_t words = (size_t)P->parts * S->lt * N;
    CROSS_CHECK_CUDA(cudaMalloc(&S->evk_a, words * 4));
    CROSS_CHECK_CUDA(cudaMalloc(&S->evk_b, words * 4));
    for (int j = 0; j < P->parts && !rc; ++j)
      for (int s = 0; s < S->lt; ++s) {
        const size_t from = ((size_t)j * LT + own[s]) * N, to = ((size_t)j * S->lt + s) * N;
        CROSS_CHECK_CUDA(cudaMemcpy(S->evk_a + to, P->evk_a + from, N * 4, cudaMemcpyDeviceToDevice));
        CROSS_CHECK_CUDA(cudaMemcpy(S->evk_b + to, P->evk_b + from, N * 4, cudaMemcpyDeviceToDevice));
      }
  }
  if (rc) {
    cross_hemul_shard_destroy(S);
    return rc;
  }
  *out = S;
  return CROSS_OK;
}

size_t cross_hemul_shard_workspace_size(cross_hemul_shard S, int64_t batch) {
  if (!S || batch < 0) return 0;
  Arena a(nullptr, 0);
  ShardBufs b;
  shard_layout(S, batch, a, b);
  return a.off;
}

int cross_hemul_shard_modup_input(cross_hemul_shard S, const uint32_t* in, int64_t B, uint32_t* cc_out, void* ws,
                                  size_t ws_bytes, void* stream) {
  CROSS_REQUIRE(S && B >= 0 && (B == 0 || (in && (cc_out || S->nq == 0))), "cross_hemul_shard_modup_input: bad argument");
  CROSS_REQUIRE((((uintptr_t)in | (uintptr_t)cc_out) & 15) == 0,
                "cross_hemul_shard_modup_input: buffers must be 16-byte aligned");
  if (B == 0 || S->nq == 0) return CROSS_OK;
  ShardBufs b;
  int rc = shard_ws_check(S, B, ws, ws_bytes, b, "cross_hemul_shard_modup_input");
  if (rc) return rc;
  const cross_hemul_plan_s* P = S->P;
  cudaStream_t st = (cudaStream_t)stream;
  const int64_t N = P->N;
  const int nq = S->nq;
  // 1. rescale of the owned limbs (ciphertext.py:267-303); in holds them at
  //    slots 0 .. nq - 1 and the last limb of Q at slot nq
  RescaleArgs ra{P->ntt_qp, P->m_last, P->m_zero, S->m_q, P->mods_dle + S->q0, P->inv_psi_last_t,
                 P->gamma_psi_t + (int64_t)S->q0 * N, P->betas + S->q0, P->thr, P->q_last, nq + 1, N};
  if ((rc = rescale_run(ra, in, (int64_t)(nq + 1) * N, b.R, b.LL, b.tmp, B * 4, st))) return rc;
  // 2. tensor product (ciphertext.py:309-324)
  const bool w32 = plan_w32(P->ntt_qp);
  const int64_t nv = N / 4;
  if (w32)
    k_tensor_lm<true><<<dim3(gx_for(nv), gy_for(B * nq)), T, 0, st>>>(b.R, b.D, B, nq, N, P->mods_dle + S->q0);
  else
    k_tensor_lm<false><<<dim3(gx_for(nv), gy_for(B * nq)), T, 0, st>>>(b.R, b.D, B, nq, N, P->mods_dle + S->q0);
  count_launch();
  // 3. INTT(d2) x psi^-i into this rank's limbs of cc (limb-outer: [limb][ct][N])
  Epi tw;
  tw.op = EPI_MUL;
  tw.tab = P->inv_psi_q_t;
  tw.trow = S->m_q;
  if ((rc = ntt_exec(P->ntt_qp, true, LP{b.D + 2 * (int64_t)nq * N, 3 * (int64_t)nq * N, N}, COEF_NATURAL,
                     LPo{cc_out, N, B * N}, COEF_TRANSPOSED, B, nq, S->m_q, tw, b.tmp, st)))
    return rc;
  CROSS_CHECK_CUDA(cudaGetLastError());
  return CROSS_OK;
}

int cross_hemul_shard_keyswitch(cross_hemul_shard S, const uint32_t* cc_all, int64_t B, uint32_t* kp_out, void* ws,
                                size_t ws_bytes, void* stream) {
  CROSS_REQUIRE(S && B >= 0 && (B == 0 || (cc_all && (kp_out || S->np == 0))), "cross_hemul_shard_keyswitch: bad argument");
  CROSS_REQUIRE((((uintptr_t)cc_all | (uintptr_t)kp_out) & 15) == 0,
                "cross_hemul_shard_keyswitch: buffers must be 16-byte aligned");
  if (B == 0 || S->lt == 0) return CROSS_OK;
  ShardBufs b;
  int rc = shard_ws_check(S, B, ws, ws_bytes, b, "cross_hemul_shard_keyswitch");
  if (rc) return rc;
  const cross_hemul_plan_s* P = S->P;
  cudaStream_t st = (cudaStream_t)stream;
  const int64_t N = P->N;
  const int nq = S->nq;
  // ModUp of every digit into the owned limbs outside it, x psi^i, NTT
  PartPtrs pp{};
  for (int j = 0; j < P->parts; ++j) {
    const int ns = S->ns[j];
    pp.e[j] = b.E[j];
    pp.ps[j] = (int64_t)ns * N;
    if (!ns) continue;
    if ((rc = bconv_run(S->ks[j], true, cc_all + (int64_t)P->dstart[j] * B * N, N, B * N, 1, b.E[j], (int64_t)ns * N,
                        N, 1, B, N, st, P->psi_qp_t, S->tgt_rows[j], S->tgt_dle[j].data())))
      return rc;
    if ((rc = ntt_exec(P->ntt_qp, false, LP{b.E[j], (int64_t)ns * N, N}, COEF_TRANSPOSED, LPo{b.E[j], (int64_t)ns * N, N},
                       COEF_NATURAL, B, ns, S->tgt_plan[j], Epi{}, b.tmp, st)))
      return rc;
  }
  // inner product with the evaluation key over the owned limbs
  if ((rc = ks_inner(plan_w32(P->ntt_qp), LP{b.D + 2 * (int64_t)nq * N, 3 * (int64_t)nq * N, N}, pp, P->parts, S->src,
                     S->lt, N, B, S->evk_a, S->evk_b, b.KS, S->mods_own, st)))
    return rc;
  // INTT of the owned P limbs of both elements x psi^-i into kp (limb-outer:
  // [limb][ct element][N])
  if (S->np > 0) {
    Epi tw;
    tw.op = EPI_MUL;
    tw.tab = P->inv_psi_p_d;
    tw.trow = S->rows_p;
    if ((rc = ntt_exec(P->ntt_p, true, LP{b.KS + (int64_t)nq * N, (int64_t)S->lt * N, N}, COEF_NATURAL,
                       LPo{kp_out, N, 2 * B * N}, P->down_layout, B * 2, S->np, S->m_p, tw, b.tmp, st)))
      return rc;
  }
  CROSS_CHECK_CUDA(cudaGetLastError());
  return CROSS_OK;
}

int cross_hemul_shard_moddown(cross_hemul_shard S, const uint32_t* kp_all, int64_t B, uint32_t* out, void* ws,
                              size_t ws_bytes, void* stream) {
  CROSS_REQUIRE(S && B >= 0 && (B == 0 || S->nq == 0 || (kp_all && out)), "cross_hemul_shard_moddown: bad argument");
  CROSS_REQUIRE((((uintptr_t)kp_all | (uintptr_t)out) & 15) == 0,
                "cross_hemul_shard_moddown: buffers must be 16-byte aligned");
  if (B == 0 || S->nq == 0) return CROSS_OK;
  ShardBufs b;
  int rc = shard_ws_check(S, B, ws, ws_bytes, b, "cross_hemul_shard_moddown");
  if (rc) return rc;
  const cross_hemul_plan_s* P = S->P;
  cudaStream_t st = (cudaStream_t)stream;
  const int64_t N = P->N;
  const int nq = S->nq;
  // BConv P -> owned Q' limbs x psi^i, then the NTT with the ModDown tail
  // (hemul.py:175-215) and the add of (d0, d1)
  if ((rc = bconv_run(S->down, true, kp_all, N, 2 * B * N, 1, b.F, (int64_t)nq * N, N, 1, B * 2, N, st, P->psi_q_d,
                      S->m_q, S->q_rows_host.data())))
    return rc;
  Epi md;
  md.op = EPI_MODDOWN;
  md.x = View{b.KS, (int64_t)S->lt * N, 0, N, 1};
  md.scal = P->pinv + S->q0;
  md.base = View{b.D, 3 * (int64_t)nq * N, (int64_t)nq * N, N, 2};
  md.base_mask = 3u;
  if ((rc = ntt_exec(P->ntt_qp, false, LP{b.F, (int64_t)nq * N, N}, P->down_layout, LPo{out, (int64_t)nq * N, N},
                     COEF_NATURAL, B * 2, nq, S->m_q, md, b.tmp, st)))
    return rc;
  CROSS_CHECK_CUDA(cudaGetLastError());
  return CROSS_OK;
}

}  // extern "C"

// ---------------------------------------------------------------------------
// Standalone steps of the HE chains (each fused inside cross_hemul /
// cross_herot), for callers that bind the reference's Ciphertext operators
// one at a time.  Element-wise, one word per thread, grid-stride.
// ---------------------------------------------------------------------------

namespace cross {
namespace {

struct ExtPtrs {
  const uint32_t* p[MAXPARTS];
};

// element e of a (rows x M) limb-innermost array or an (outer x M x n)
// limb-major one: its limb index
template <bool LM>
__device__ __forceinline__ int limb_of(int64_t e, int M, int64_t n) {
  return LM ? (int)((e / n) % M) : (int)(e % M);
}

template <bool LM>
__global__ void k_ks_inner_any(ExtPtrs ext, int dnum, const uint32_t* __restrict__ evka, const uint32_t* __restrict__ evkb,
                               uint32_t* __restrict__ out, int64_t batch, int64_t n, int M,
                               const ModC* __restrict__ mods) {
  const int64_t per = n * M, total = batch * per;
  for (int64_t e = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; e < total; e += (int64_t)gridDim.x * blockDim.x) {
    const int64_t b = e / per, w = e - b * per;   // w: position inside one ciphertext element
    uint64_t s0 = 0, s1 = 0;
    for (int j = 0; j < dnum; ++j) {
      const uint64_t x = ext.p[j][e];
      s0 += x * evkb[(int64_t)j * per + w];
      s1 += x * evka[(int64_t)j * per + w];
    }
    const ModC mc = mods[limb_of<LM>(w, M, n)];
    out[b * 2 * per + w] = barrett_any(s0, mc);
    out[b * 2 * per + per + w] = barrett_any(s1, mc);
  }
}

__global__ void k_moddown_sub_mul(const uint32_t* __restrict__ x, const uint32_t* __restrict__ y,
                                  const uint32_t* __restrict__ pinv, const uint32_t* __restrict__ base,
                                  uint32_t* __restrict__ out, int64_t rows, int M, const ModC* __restrict__ mods) {
  const int64_t total = rows * M;
  for (int64_t e = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; e < total; e += (int64_t)gridDim.x * blockDim.x) {
    const int l = (int)(e % M);
    const ModC mc = mods[l];
    const uint32_t q = (uint32_t)mc.q, a = x[e], b = y[e];
    const uint32_t s = a < b ? a + q - b : a - b;                 // uint32 wrap, hemul.py:199-203
    uint32_t t = barrett_any((uint64_t)s * pinv[l], mc);          // modmul(PInvModq), hemul.py:205-206
    if (base) {
      const uint32_t v = base[e] + t;                             // hemul.py:214-215
      t = v >= q ? v - q : v;
    }
    out[e] = t;
  }
}

template <bool LM>
__global__ void k_rescale_lift_any(const uint32_t* __restrict__ last, uint32_t q_last, uint32_t thr,
                                   const uint32_t* __restrict__ gpsi, uint32_t* __restrict__ out, int64_t polys,
                                   int64_t n, int M, const ModC* __restrict__ mods) {
  const int64_t per = n * M, total = polys * per;
  for (int64_t e = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; e < total; e += (int64_t)gridDim.x * blockDim.x) {
    const int64_t p = e / per, w = e - p * per;
    const int l = limb_of<LM>(w, M, n);
    const int64_t t = LM ? w % n : w / M;
    const ModC mc = mods[l];
    const uint32_t a = last[p * n + t];
    const uint64_t lifted = a < thr ? (uint64_t)a : mc.q - (uint64_t)q_last + (uint64_t)a;   // ciphertext.py:285-290
    out[e] = barrett_any(lifted * gpsi[w], mc);                                           // :291-295
  }
}

unsigned ew_grid(int64_t total) {
  const int64_t g = (total + T - 1) / T;
  const int64_t cap = (int64_t)device_sm_count() * 16;
  return (unsigned)(g < 1 ? 1 : (g > cap ? cap : g));
}

}  // namespace
}  // namespace cross

extern "C" {

int cross_ks_inner_product(cross_moduli moduli, const uint32_t* const* ext, int dnum, const uint32_t* evk_a,
                           const uint32_t* evk_b, uint32_t* out, int64_t batch, int64_t n, int layout, void* stream) {
  CROSS_REQUIRE(moduli && ext && evk_a && evk_b && out && batch >= 0 && n >= 1,
                "cross_ks_inner_product: bad argument");
  CROSS_REQUIRE(dnum >= 1 && dnum <= MAXPARTS, "cross_ks_inner_product: dnum=%d out of range 1..%d", dnum, MAXPARTS);
  CROSS_REQUIRE(layout == CROSS_LAYOUT_REFERENCE || layout == CROSS_LAYOUT_LIMB_MAJOR,
                "cross_ks_inner_product: unknown layout %d", layout);
  if (batch == 0) return CROSS_OK;
  ExtPtrs e{};
  for (int j = 0; j < dnum; ++j) {
    CROSS_REQUIRE(ext[j], "cross_ks_inner_product: ext[%d] is null", j);
    e.p[j] = ext[j];
  }
  const int M = moduli->n;
  const int64_t total = batch * n * M;
  cudaStream_t st = (cudaStream_t)stream;
  if (layout == CROSS_LAYOUT_LIMB_MAJOR)
    k_ks_inner_any<true><<<ew_grid(total), T, 0, st>>>(e, dnum, evk_a, evk_b, out, batch, n, M, moduli->dev);
  else
    k_ks_inner_any<false><<<ew_grid(total), T, 0, st>>>(e, dnum, evk_a, evk_b, out, batch, n, M, moduli->dev);
  count_launch();
  CROSS_CHECK_CUDA(cudaGetLastError());
  return CROSS_OK;
}

int cross_moddown_sub_mul(cross_moduli moduli, const uint32_t* x, const uint32_t* y, const uint32_t* p_inv_mod_q,
                          const uint32_t* base, uint32_t* out, int64_t rows, void* stream) {
  CROSS_REQUIRE(moduli && x && y && p_inv_mod_q && out && rows >= 0, "cross_moddown_sub_mul: bad argument");
  if (rows == 0) return CROSS_OK;
  const int64_t total = rows * moduli->n;
  k_moddown_sub_mul<<<ew_grid(total), T, 0, (cudaStream_t)stream>>>(x, y, p_inv_mod_q, base, out, rows, moduli->n,
                                                                   moduli->dev);
  count_launch();
  CROSS_CHECK_CUDA(cudaGetLastError());
  return CROSS_OK;
}

int cross_rescale_lift(cross_moduli moduli, const uint32_t* last, uint32_t q_last, const uint32_t* gamma_psi,
                       uint32_t* out, int64_t polys, int64_t n, int layout, void* stream) {
  CROSS_REQUIRE(moduli && last && gamma_psi && out && polys >= 0 && n >= 1 && q_last >= 3,
                "cross_rescale_lift: bad argument");
  CROSS_REQUIRE(layout == CROSS_LAYOUT_REFERENCE || layout == CROSS_LAYOUT_LIMB_MAJOR,
                "cross_rescale_lift: unknown layout %d", layout);
  for (const ModC& mc : moduli->host)
    CROSS_REQUIRE(mc.q + 1 > q_last, "cross_rescale_lift: target modulus %llu below q_last - 1",
                  (unsigned long long)mc.q);
  if (polys == 0) return CROSS_OK;
  const int M = moduli->n;
  const int64_t total = polys * n * M;
  const uint32_t thr = (q_last + 1) / 2;                          // ciphertext.py:260
  cudaStream_t st = (cudaStream_t)stream;
  if (layout == CROSS_LAYOUT_LIMB_MAJOR)
    k_rescale_lift_any<true><<<ew_grid(total), T, 0, st>>>(last, q_last, thr, gamma_psi, out, polys, n, M, moduli->dev);
  else
    k_rescale_lift_any<false><<<ew_grid(total), T, 0, st>>>(last, q_last, thr, gamma_psi, out, polys, n, M, moduli->dev);
  count_launch();
  CROSS_CHECK_CUDA(cudaGetLastError());
  return CROSS_OK;
}

}  // extern "C"
