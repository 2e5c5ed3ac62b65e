// Basis conversion (bconv.py:173-252).
//
// basis_change_bat: c_i = Barrett_src_i(x_i * QHatInvModq_i); then for every
// target limb j the BAT contraction
//   S_j = sum_b ( sum_{i,a} byte_a(c_i) * QHatModpBAT[(i,a), j, b] ) << 8b
// and out_j = Barrett_dst_j(S_j).  The inner sum over the four bytes a of one
// c_i is one dp4a against the packed BAT column.
// basis_change: S_j = sum_i c_i * QHatModp[i, j] in uint64, then Barrett.
//
// Two kernels compute basis_change_bat.  k_bconv_tc (contiguous coefficients,
// n % 128 == 0) runs the contraction on the tensor cores: for 128 coefficients
// t, A[t][(i, a)] = byte_a(c_i[t]) (K = 4 sq bytes) against
// B[(j, b)][(i, a)] = QHatModpBAT[(i, a), j, b] (N = 4 sp), one
// tcgen05.mma.kind::i8 per 8 source limbs, and the epilogue recombines the four
// byte planes b of every target limb.  k_bconv (any strides) uses dp4a.
#include <cstdlib>
#include <type_traits>
#include <vector>

#include "internal.hpp"
#include "tc_ptx.cuh"

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

// ---------------------------------------------------------------------------
// Tensor-core basis conversion.  One CTA of 256 threads per tile of 128
// coefficients of one polynomial, two threads per coefficient row t (TMEM lane
// t), each taking half of the source and half of the target limbs:
//   1. c_i = Barrett_src_i(x_i[t] * QHatInvModq_i) written as row t of the
//      K-major A tile (no swizzle: 8-row x 16-byte core matrices, K halves 128 B
//      apart, 8-row groups 256 B apart; one 16-byte store per 4 limbs);
//   2. thread 0 issues kb MMAs (M = 128, N = nn, K = 32) into TMEM and commits;
//   3. every thread reads its half of the accumulator row and writes
//      out_j[t] = Barrett_dst_j(sum_b D[t][4j + b] << 8b) (times the psi twist).
// The B image (QHatModpBAT in the same core-matrix layout) and the per-limb
// constants stay in shared memory.  The MMA completion wait is bounded; on
// expiry the kernel records code 21 in the plan's error word and stops.
constexpr int BT_ROWS = 128;      // coefficients per tile (TMEM lanes)
constexpr int BT_THREADS = 256;   // two threads per coefficient row
using namespace tc;

struct BconvTcArgs {
  const uint32_t* in;
  int64_t in_ps, in_ls;
  uint32_t* out;
  int64_t out_ps, out_ls;
  int polys, n, sq, sp, kb, nn;
  uint32_t tmem_cols;
  const ModC* src;
  const ModC* dst;
  const uint32_t* qhat_inv;
  const uint8_t* bimg;
  const uint32_t* twist;
  const uint16_t* trow;
  int* err;
  bool src_fast;  // reduce_fast is exact for every source modulus
};

__device__ __forceinline__ uint64_t kmajor_desc(uint32_t addr) {
  // start >> 4, leading (K) byte offset 128 >> 4, stride (8-row) byte offset
  // 256 >> 4, descriptor version 1, layout SWIZZLE_NONE
  return (uint64_t)((addr >> 4) & 0x3FFF) | ((uint64_t)(128 >> 4) << 16) | ((uint64_t)(256 >> 4) << 32) |
         ((uint64_t)1 << 46);
}

// NN: compile-time polynomial length with unit-stride limb rows (in_ls = out_ls
// = n = NN), so tile arithmetic and store offsets are immediates; 0 = run time.
template <bool FAST, bool TWIST, int KB, int SPMAX, int NN>
__global__ void __launch_bounds__(BT_THREADS, 4) k_bconv_tc(const BconvTcArgs a) {
  extern __shared__ uint8_t sm_raw[];
  uint8_t* As = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(sm_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* Bs = As + a.kb * 4096;
  uint64_t* bar = reinterpret_cast<uint64_t*>(Bs + a.kb * (a.nn / 8) * 256);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bar + 1);
  volatile int& abort = *reinterpret_cast<volatile int*>(tmem_slot + 1);
  uint4* dc = reinterpret_cast<uint4*>(tmem_slot + 2);   // [sp] target {q, m, s_w, twist row}
  const uint32_t** tp = reinterpret_cast<const uint32_t**>(dc + a.sp);   // [sp] twist row of each target limb
  ModC* sc = reinterpret_cast<ModC*>(tp + a.sp);          // [sq] source moduli
  uint32_t* shi = reinterpret_cast<uint32_t*>(sc + a.sq);        // [sq] QHatInvModq
  const int t = threadIdx.x, warp = t >> 5;
  const int n = NN ? NN : a.n;
  const int64_t in_ls = NN ? NN : a.in_ls, out_ls = NN ? NN : a.out_ls;

  for (int i = t; i < a.kb * (a.nn / 8) * 16; i += BT_THREADS)
    reinterpret_cast<uint4*>(Bs)[i] = reinterpret_cast<const uint4*>(a.bimg)[i];
  for (int j = t; j < a.sp; j += BT_THREADS) {
    dc[j] = make_uint4((uint32_t)a.dst[j].q, (uint32_t)a.dst[j].m, a.dst[j].s_w, TWIST ? a.trow[j] : 0u);
    tp[j] = TWIST ? a.twist + (int64_t)a.trow[j] * n : nullptr;
  }
  for (int i = t; i < a.sq; i += BT_THREADS) {
    sc[i] = a.src[i];
    shi[i] = a.qhat_inv[i];
  }
  if (t == 0) {
    mbar_init(bar, 1);
    abort = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(saddr(tmem_slot)),
                 "r"(a.tmem_cols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const uint32_t idesc = (2u << 4) | ((uint32_t)(a.nn >> 3) << 17) | ((uint32_t)(BT_ROWS >> 4) << 24);
  const int tiles_pp = n / BT_ROWS;
  const int total = a.polys * tiles_pp;
  // Thread (row, h): coefficient row = TMEM lane, half h of the work.  It packs
  // the source limbs 4g..4g+3 for the K-halves g = 2gi + h, and produces the
  // target limbs [h * SPMAX/2, (h + 1) * SPMAX/2).
  const int row = t & (BT_ROWS - 1), h = t / BT_ROWS;
  constexpr int JH = SPMAX / 2;
  // inputs of the next tile, loaded while the current one is converted
  uint32_t xin[4 * KB];
  auto load_inputs = [&](int w) {
    const int poly = w / tiles_pp;
    const uint32_t* x = a.in + (int64_t)poly * a.in_ps + (w - poly * tiles_pp) * BT_ROWS + row;
#pragma unroll
    for (int gi = 0; gi < KB; ++gi)
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int i = 4 * (2 * gi + h) + e;
        xin[4 * gi + e] = i < a.sq ? __ldg(x + (int64_t)i * in_ls) : 0u;
      }
  };
  if ((int)blockIdx.x < total) load_inputs(blockIdx.x);
  uint32_t phase = 0;
  for (int w = blockIdx.x; w < total; w += gridDim.x) {
    const int poly = w / tiles_pp;
    const int t0 = (w - poly * tiles_pp) * BT_ROWS;
    // 1. source residues, 4 limbs (16 bytes of K) per store
#pragma unroll
    for (int gi = 0; gi < KB; ++gi) {
      if (gi < a.kb) {
        const int g = 2 * gi + h;
        uint32_t c[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int i = 4 * g + e;
          uint32_t v = 0;
          if (i < a.sq) {
            const uint32_t xv = xin[4 * gi + e], hv = shi[i];
            // x < 2^31 and QHatInv < q keep the product below 2^31 q, where the
            // fast form is exact (always so for transform outputs)
            if (FAST && a.src_fast && xv < 0x80000000u)
              v = reduce_fast2(xv * hv, __umulhi(xv, hv), (uint32_t)sc[i].q, (uint32_t)sc[i].m, sc[i].s_w);
            else if (FAST)
              v = barrett_w32((uint64_t)xv * hv, (uint32_t)sc[i].q, (uint32_t)sc[i].m, sc[i].s_w);
            else
              v = barrett((uint64_t)xv * hv, sc[i]);
          }
          c[e] = v;
        }
        *reinterpret_cast<uint4*>(As + gi * 4096 + (row >> 3) * 256 + h * 128 + (row & 7) * 16) =
            make_uint4(c[0], c[1], c[2], c[3]);
      }
    }
    if (w + (int)gridDim.x < total) load_inputs(w + gridDim.x);
    // twist factors of this tile, in flight during the MMA
    uint32_t tw[JH];
    if (TWIST) {
#pragma unroll
      for (int jj = 0; jj < JH; ++jj) {
        const int j = h * JH + jj;
        tw[jj] = j < a.sp ? __ldg(tp[j] + t0 + row) : 0u;
      }
    }
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    tc_fence_before();
    __syncthreads();
    bool ok = true;
    if (t == 0) {
      tc_fence_after();
      for (int k = 0; k < a.kb; ++k) {
        const uint64_t ad = kmajor_desc(saddr(As + k * 4096));
        const uint64_t bd = kmajor_desc(saddr(Bs + k * (a.nn / 8) * 256));
        const uint32_t acc = k > 0, z = 0;
        asm volatile(
            "{\n\t.reg .pred p;\n\t"
            "setp.ne.b32 p, %4, 0;\n\t"
            "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, {%5, %5, %5, %5}, p;\n\t}\n" ::"r"(tmem),
            "l"(ad), "l"(bd), "r"(idesc), "r"(acc), "r"(z));
      }
      asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(saddr(bar))
                   : "memory");
      // 2. accumulator ready (one waiting thread; the others sleep in the barrier)
      ok = mbar_wait(bar, phase, abort, a.err, 21);
    }
    phase ^= 1;
    if (__syncthreads_or(!ok)) break;
    tc_fence_after();
    // 3. four target limbs per 16 accumulator columns, this half's limbs only
    uint32_t* y = a.out + (int64_t)poly * a.out_ps + t0 + row;
#pragma unroll
    for (int qc = 0; qc < JH / 4; ++qc) {
      const int j0 = h * JH + 4 * qc;
      if (4 * j0 < a.nn) {
        uint32_t v[16];
        tmem_ld16(tmem + ((uint32_t)((warp & 3) * 32) << 16) + 4 * j0, v);
#pragma unroll
        for (int jj = 0; jj < 4; ++jj) {
          const int j = j0 + jj;
          if (j < a.sp) {
            const uint4 cj = dc[j];
            const uint32_t q = cj.x, m = cj.y, sw = cj.z;
            const uint64_t z = combine4_mad(v[4 * jj], v[4 * jj + 1], v[4 * jj + 2], v[4 * jj + 3]);
            const uint32_t twj = tw[4 * qc + jj];
            uint32_t r;
            if (FAST) {
              r = reduce_fast(z, q, m, sw);
              if (TWIST) r = reduce_fast2(r * twj, __umulhi(r, twj), q, m, sw);
            } else {
              const ModC mc = a.dst[j];
              r = barrett(z, mc);
              if (TWIST) r = barrett((uint64_t)r * twj, mc);
            }
            y[(int64_t)j * out_ls] = r;
          }
        }
      }
    }
    tc_fence_before();
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0)
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(a.tmem_cols) : "memory");
}

// Shared memory of one k_bconv_tc CTA: the A and B tiles plus constants,
// padded so that no more CTAs fit on an SM (sm_bytes of shared memory, 1 KiB
// reserved per CTA) than its 512 TMEM columns serve.  0 when impossible.
size_t bconv_tc_smem(int sq, int sp, int kb, int nn, uint32_t tmem_cols, size_t sm_bytes, int* ctas_per_sm) {
  const size_t need = 1024 + (size_t)kb * 4096 + (size_t)kb * (nn / 8) * 256 + 16 + (size_t)sp * (16 + 8) +
                      (size_t)sq * (sizeof(ModC) + 4);
  const int ctas = (int)(512 / tmem_cols);
  // (ctas + 1) CTAs of s + 1 KiB each must not fit, ctas of them must
  const size_t lo = sm_bytes / (ctas + 1), hi = sm_bytes / ctas - 1024;
  if (lo + 64 > hi) return 0;
  size_t s = (lo + hi) / 2;
  if (s < need) s = need;
  *ctas_per_sm = ctas;
  return (s > hi) ? 0 : s;
}

template <bool FAST, bool TWIST, int KB, int SPMAX, int NN>
int launch_bconv_tc(const BconvTcArgs& a, size_t smem, int ctas_per_sm, cudaStream_t st) {
  const int sms = device_sm_count();
  auto kern = k_bconv_tc<FAST, TWIST, KB, SPMAX, NN>;
  CROSS_CHECK_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
  const int64_t total = (int64_t)a.polys * (a.n / BT_ROWS);
  const int64_t cap = (int64_t)sms * ctas_per_sm;
  kern<<<(unsigned)(total < cap ? total : cap), BT_THREADS, smem, st>>>(a);
  count_launch();
  CROSS_CHECK_CUDA(cudaGetLastError());
  return CROSS_OK;
}

template <bool FAST, bool TWIST>
int launch_bconv_tc_any(const BconvTcArgs& a, size_t smem, int ctas_per_sm, cudaStream_t st) {
  const bool n64k = a.n == 65536 && a.in_ls == 65536 && a.out_ls == 65536;
  if (a.kb == 1 && a.sp <= 24)
    return n64k ? launch_bconv_tc<FAST, TWIST, 1, 24, 65536>(a, smem, ctas_per_sm, st)
                : launch_bconv_tc<FAST, TWIST, 1, 24, 0>(a, smem, ctas_per_sm, st);
  if (a.kb == 1) return launch_bconv_tc<FAST, TWIST, 1, 64, 0>(a, smem, ctas_per_sm, st);
  return launch_bconv_tc<FAST, TWIST, 4, 64, 0>(a, smem, ctas_per_sm, st);
}

// ---------------------------------------------------------------------------
// Tensor-core basis conversion with every per-limb constant in the kernel's
// parameter space (k_bconv_tcc).  Same tile structure as k_bconv_tc -- a CTA
// of 256 threads per tile of 128 coefficients, thread (row, h) packs the source
// limb groups 2k + h and produces the target limbs [h JH, (h + 1) JH) -- but the
// half h is a template argument of the per-thread work, so every limb index is
// a compile-time constant: the moduli, Barrett constants, QHatInvModq and twist
// rows are read from the constant bank as instruction operands, the limb-row
// strides of the N = 2^16 instantiation are immediates, and the byte planes
// are recombined in two 32-bit multiply-adds and one widening one (every BAT
// sum of at most 32 source limbs is below 2^23).  Used when every source and
// target modulus passes reduce_fast_ok (all moduli of the HE parameter sets).
// Per-limb constants.  Barrett plans: m and s_w in the second and third
// arrays.  Montgomery: q^-1 mod 2^32 in the second.  BAT-lazy: the words
// 2^(32 + 8i) mod q, i = 0..3, in the second, third and the two extra arrays.
struct BconvConsts {
  uint32_t sq_q[32], sq_m[32], sq_sw[32], sq_hi[32];   // source q_i, Barrett m, s_w, QHatInvModq_i
  uint32_t sq_r2[32], sq_r3[32];                       // source BAT-lazy words 2, 3
  uint32_t dq[64], dm[64], dsw[64];                    // target q_j, Barrett m, s_w
  uint32_t dr2[64], dr3[64];                           // target BAT-lazy words 2, 3
  const uint32_t* tp[64];                              // twist row of target j (TWIST)
};

struct BconvTccArgs {
  const uint32_t* in;
  int64_t in_ps, in_ls;
  void* out;                        // uint64 elements for BAT-lazy plans, else uint32
  int64_t out_ps, out_ls;
  int polys, n, sq, sp, kb, nn;
  uint32_t tmem_cols;
  const uint8_t* bimg;
  int* err;
  BconvConsts k;
};

// sum_p a_p << 8p (bconv.py:31-37) for a_p < 2^23: a0 + a1 2^8 and a2 + a3 2^8
// fit 32 bits, and the sum is their first plus 2^16 times the second.
__device__ __forceinline__ uint64_t combine4_small(uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3) {
  const uint32_t s = a0 + (a1 << 8), u = a2 + (a3 << 8);
  return (uint64_t)s + ((uint64_t)u << 16);
}

template <int H, int KB, int NN>
__device__ __forceinline__ void bcc_load(const BconvTccArgs& a, int w, int tiles_pp, int row, uint32_t (&xin)[4 * KB]) {
  const int64_t in_ls = NN ? NN : a.in_ls;
  const int poly = w / tiles_pp;
  const uint32_t* x = a.in + (int64_t)poly * a.in_ps + (w - poly * tiles_pp) * BT_ROWS + row;
#pragma unroll
  for (int k = 0; k < KB; ++k)
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const int i = 4 * (2 * k + H) + e;
      xin[4 * k + e] = i < a.sq ? __ldg(x + (int64_t)i * in_ls) : 0u;
    }
}

// c_i = Barrett_i(x_i QHatInvModq_i) of this thread's source groups (the
// exact 32-bit form for x < 2^31, where x QHatInv < 2^31 q; the 64-bit form
// above), and their store as row `row` of the K-major A tile.
template <int H, int KB, int RED>
__device__ __forceinline__ void bcc_reduce(const BconvTccArgs& a, const uint32_t (&xin)[4 * KB], uint32_t (&c)[4 * KB]) {
#pragma unroll
  for (int k = 0; k < KB; ++k) {
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const int i = 4 * (2 * k + H) + e;
      uint32_t v = 0;
      if (k < a.kb && i < a.sq) {
        const uint32_t xv = xin[4 * k + e], hv = a.k.sq_hi[i], q = a.k.sq_q[i], m = a.k.sq_m[i],
                       sw = a.k.sq_sw[i];
        if (RED == RED_MONTGOMERY) {
          v = montgomery((uint64_t)xv * hv, q, m);                       // bconv.py:273
        } else if (RED == RED_BAT_LAZY) {
          const uint32_t r[4] = {m, sw, a.k.sq_r2[i], a.k.sq_r3[i]};
          v = (uint32_t)bat_lazy((uint64_t)xv * hv, r) % q;             // bconv.py:382-386
        } else {
          v = xv < 0x80000000u ? reduce_fast2(xv * hv, __umulhi(xv, hv), q, m, sw)
                               : barrett_w32((uint64_t)xv * hv, q, m, sw);
        }
      }
      c[4 * k + e] = v;
    }
  }
}
template <int H, int KB>
__device__ __forceinline__ void bcc_write(const BconvTccArgs& a, uint8_t* As, int row, const uint32_t (&c)[4 * KB]) {
#pragma unroll
  for (int k = 0; k < KB; ++k)
    if (k < a.kb)
      *reinterpret_cast<uint4*>(As + k * 4096 + (row >> 3) * 256 + H * 128 + (row & 7) * 16) =
          make_uint4(c[4 * k], c[4 * k + 1], c[4 * k + 2], c[4 * k + 3]);
}

template <int H, int JH, bool TWIST>
__device__ __forceinline__ void bcc_twist(const BconvTccArgs& a, int t, uint32_t (&tw)[JH]) {
  if (TWIST) {
#pragma unroll
    for (int jj = 0; jj < JH; ++jj) {
      const int j = H * JH + jj;
      tw[jj] = j < a.sp ? __ldg(a.k.tp[j] + t) : 0u;
    }
  }
}

// out_j[t] = Barrett_j(sum_b D[t][4j + b] << 8b) (x psi twist) for this
// thread's targets; lane quadrant (warp & 3) of the accumulator.
template <int H, int JH, bool TWIST, int NN, int RED>
__device__ __forceinline__ void bcc_store(const BconvTccArgs& a, uint32_t tmem, int warp, int64_t yoff,
                                          const uint32_t (&tw)[JH]) {
  const int64_t out_ls = NN ? NN : a.out_ls;
#pragma unroll
  for (int qc = 0; qc < JH / 4; ++qc) {
    constexpr int J0 = H * JH;
    const int j0 = J0 + 4 * qc;
    if (4 * j0 < a.nn) {
      uint32_t v[16];
      tmem_ld16(tmem + ((uint32_t)((warp & 3) * 32) << 16) + 4 * j0, v);
#pragma unroll
      for (int jj = 0; jj < 4; ++jj) {
        const int j = j0 + jj;
        if (j < a.sp) {
          const uint32_t q = a.k.dq[j], m = a.k.dm[j], sw = a.k.dsw[j];
          const uint64_t z = combine4_small(v[4 * jj], v[4 * jj + 1], v[4 * jj + 2], v[4 * jj + 3]);
          if (RED == RED_BAT_LAZY) {
            const uint32_t r4[4] = {m, sw, a.k.dr2[j], a.k.dr3[j]};
            static_cast<uint64_t*>(a.out)[yoff + (int64_t)j * out_ls] = bat_lazy(z, r4);   // bconv.py:368
          } else {
            uint32_t r;
            if (RED == RED_MONTGOMERY) {
              r = montgomery(z, q, m);                                       // bconv.py:288
            } else {
              r = reduce_fast(z, q, m, sw);
              if (TWIST) {
                const uint32_t twj = tw[4 * qc + jj];
                r = reduce_fast2(r * twj, __umulhi(r, twj), q, m, sw);
              }
            }
            static_cast<uint32_t*>(a.out)[yoff + (int64_t)j * out_ls] = r;
          }
        }
      }
    }
  }
}

template <bool TWIST, int KB, int SPMAX, int NN, int RED>
__global__ void __launch_bounds__(BT_THREADS, 4) k_bconv_tcc(const __grid_constant__ BconvTccArgs a) {
  extern __shared__ uint8_t sm_raw[];
  uint8_t* As = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(sm_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* Bs = As + a.kb * 4096;
  uint64_t* bar = reinterpret_cast<uint64_t*>(Bs + a.kb * (a.nn / 8) * 256);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bar + 1);
  volatile int& abort = *reinterpret_cast<volatile int*>(tmem_slot + 1);
  constexpr int JH = SPMAX / 2;
  const int t = threadIdx.x, warp = t >> 5;
  const int row = t & (BT_ROWS - 1), h = t / BT_ROWS;   // h is uniform per warp
  const int n = NN ? NN : a.n;
  for (int i = t; i < a.kb * (a.nn / 8) * 16; i += BT_THREADS)
    reinterpret_cast<uint4*>(Bs)[i] = reinterpret_cast<const uint4*>(a.bimg)[i];
  if (t == 0) {
    mbar_init(bar, 1);
    abort = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(saddr(tmem_slot)),
                 "r"(a.tmem_cols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const uint32_t idesc = (2u << 4) | ((uint32_t)(a.nn >> 3) << 17) | ((uint32_t)(BT_ROWS >> 4) << 24);
  const int tiles_pp = n / BT_ROWS;
  const int total = a.polys * tiles_pp;
  // SHADOW (one source group): the next tile's reductions run while the MMA
  // of this tile is in flight, and its inputs are loaded a tile further ahead
  constexpr bool SHADOW = KB == 1;
  uint32_t xin[4 * KB], cv[4 * KB];
  uint32_t tw[JH];
  const int g = (int)gridDim.x;
  if ((int)blockIdx.x < total) {
    if (h == 0) bcc_load<0, KB, NN>(a, blockIdx.x, tiles_pp, row, xin);
    else bcc_load<1, KB, NN>(a, blockIdx.x, tiles_pp, row, xin);
    if (SHADOW) {
      if (h == 0) bcc_reduce<0, KB, RED>(a, xin, cv);
      else bcc_reduce<1, KB, RED>(a, xin, cv);
      if ((int)blockIdx.x + g < total) {
        if (h == 0) bcc_load<0, KB, NN>(a, blockIdx.x + g, tiles_pp, row, xin);
        else bcc_load<1, KB, NN>(a, blockIdx.x + g, tiles_pp, row, xin);
      }
    }
  }
  uint32_t phase = 0;
  for (int w = blockIdx.x; w < total; w += g) {
    const int poly = w / tiles_pp;
    const int t0 = (w - poly * tiles_pp) * BT_ROWS;
    // 1. source residues into the A tile, then the next tile's inputs and
    //    this tile's twists, in flight during the MMA
    const bool more = w + g < total;
    if (!SHADOW) {
      if (h == 0) bcc_reduce<0, KB, RED>(a, xin, cv);
      else bcc_reduce<1, KB, RED>(a, xin, cv);
    }
    if (h == 0) {
      bcc_write<0, KB>(a, As, row, cv);
      if (more && !SHADOW) bcc_load<0, KB, NN>(a, w + g, tiles_pp, row, xin);
      bcc_twist<0, JH, TWIST>(a, t0 + row, tw);
    } else {
      bcc_write<1, KB>(a, As, row, cv);
      if (more && !SHADOW) bcc_load<1, KB, NN>(a, w + g, tiles_pp, row, xin);
      bcc_twist<1, JH, TWIST>(a, t0 + row, tw);
    }
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    tc_fence_before();
    __syncthreads();
    bool ok = true;
    if (t == 0) {
      tc_fence_after();
      for (int k = 0; k < a.kb; ++k) {
        const uint64_t ad = kmajor_desc(saddr(As + k * 4096));
        const uint64_t bd = kmajor_desc(saddr(Bs + k * (a.nn / 8) * 256));
        const uint32_t acc = k > 0, z = 0;
        asm volatile(
            "{\n\t.reg .pred p;\n\t"
            "setp.ne.b32 p, %4, 0;\n\t"
            "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, {%5, %5, %5, %5}, p;\n\t}\n" ::"r"(tmem),
            "l"(ad), "l"(bd), "r"(idesc), "r"(acc), "r"(z));
      }
      asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(saddr(bar))
                   : "memory");
    }
    if (SHADOW && more) {
      // the next tile's reductions (registers only: the MMA reads the A tile)
      // and the inputs of the tile after it
      if (h == 0) bcc_reduce<0, KB, RED>(a, xin, cv);
      else bcc_reduce<1, KB, RED>(a, xin, cv);
      if (w + 2 * g < total) {
        if (h == 0) bcc_load<0, KB, NN>(a, w + 2 * g, tiles_pp, row, xin);
        else bcc_load<1, KB, NN>(a, w + 2 * g, tiles_pp, row, xin);
      }
    }
    // 2. accumulator ready (one waiting thread; the others sleep in the barrier)
    if (t == 0) ok = mbar_wait(bar, phase, abort, a.err, 22);
    phase ^= 1;
    if (__syncthreads_or(!ok)) break;
    tc_fence_after();
    // 3. this half's target limbs
    const int64_t yoff = (int64_t)poly * a.out_ps + t0 + row;
    if (h == 0) bcc_store<0, JH, TWIST, NN, RED>(a, tmem, warp, yoff, tw);
    else bcc_store<1, JH, TWIST, NN, RED>(a, tmem, warp, yoff, tw);
    tc_fence_before();
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0)
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(a.tmem_cols) : "memory");
}

template <bool TWIST, int KB, int SPMAX, int NN, int RED>
int launch_bconv_tcc(const BconvTccArgs& a, size_t smem, int ctas_per_sm, cudaStream_t st) {
  const int sms = device_sm_count();
  auto kern = k_bconv_tcc<TWIST, KB, SPMAX, NN, RED>;
  CROSS_CHECK_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
  const int64_t total = (int64_t)a.polys * (a.n / BT_ROWS);
  const int64_t cap = (int64_t)sms * ctas_per_sm;
  kern<<<(unsigned)(total < cap ? total : cap), BT_THREADS, smem, st>>>(a);
  count_launch();
  CROSS_CHECK_CUDA(cudaGetLastError());
  return CROSS_OK;
}

template <bool TWIST, int RED = RED_BARRETT_FAST>
int launch_bconv_tcc_any(const BconvTccArgs& a, size_t smem, int ctas_per_sm, cudaStream_t st) {
  const bool n64k = a.n == 65536 && a.in_ls == 65536 && a.out_ls == 65536;
#define CROSS_BCC(KB, SPM)                                                                        \
  return n64k ? launch_bconv_tcc<TWIST, KB, SPM, 65536, RED>(a, smem, ctas_per_sm, st)            \
              : launch_bconv_tcc<TWIST, KB, SPM, 0, RED>(a, smem, ctas_per_sm, st)
  if (a.kb == 1 && a.sp <= 24) CROSS_BCC(1, 24);
  if (a.kb == 1 && a.sp <= 40) CROSS_BCC(1, 40);
  if (a.kb == 1) CROSS_BCC(1, 64);
  if (a.kb <= 2 && a.sp <= 40) CROSS_BCC(2, 40);
  if (a.kb <= 3 && a.sp <= 40) CROSS_BCC(3, 40);
  CROSS_BCC(4, 64);
#undef CROSS_BCC
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

// basis_change_bat of a Montgomery or BAT-lazy plan on the tensor cores
// (contiguous coefficients, n % 128 == 0): the same BAT contraction as
// Barrett with the context's input scaling and output reduction (bconv.py:
// 234-246 with MontgomeryContext / BATLazyContext.modular_reduction).  Returns
// CROSS_ERR_UNSUPPORTED (nothing launched) when the shape does not qualify.
int bconv_var_tc(const cross_bconv_plan_s* P, const uint32_t* in, int64_t in_ps, int64_t in_ls, int64_t in_ts,
                 void* out, int64_t out_ps, int64_t out_ls, int64_t out_ts, int64_t polys, int64_t n,
                 cudaStream_t st) {
  if (!P->tc_bimg || in_ts != 1 || out_ts != 1 || n % BT_ROWS != 0 || polys * (n / BT_ROWS) >= (1ll << 31) ||
      (P->red != CROSS_REDUCTION_MONTGOMERY && P->red != CROSS_REDUCTION_BAT_LAZY) ||
      (int)P->src_v_host.size() != P->sq || (int)P->dst_v_host.size() != P->sp)
    return CROSS_ERR_UNSUPPORTED;
  BconvTccArgs c{in, in_ps, in_ls, out, out_ps, out_ls, (int)polys, (int)n, P->sq, P->sp, P->tc_kb, P->tc_nn,
                 64, P->tc_bimg, P->err, {}};
  while ((int)c.tmem_cols < c.nn) c.tmem_cols <<= 1;
  int cpsm = 0;
  const size_t smc = bconv_tc_smem(P->sq, P->sp, P->tc_kb, P->tc_nn, c.tmem_cols, (size_t)device_smem_per_sm(), &cpsm);
  if (!smc) return CROSS_ERR_UNSUPPORTED;
  const bool mont = P->red == CROSS_REDUCTION_MONTGOMERY;
  for (int i = 0; i < P->sq; ++i) {
    const VarC& v = P->src_v_host[i];
    c.k.sq_q[i] = v.q;
    c.k.sq_hi[i] = P->qhat_inv_host[i];
    c.k.sq_m[i] = mont ? v.qinv : v.r[0];
    c.k.sq_sw[i] = v.r[1];
    c.k.sq_r2[i] = v.r[2];
    c.k.sq_r3[i] = v.r[3];
  }
  for (int j = 0; j < P->sp; ++j) {
    const VarC& v = P->dst_v_host[j];
    c.k.dq[j] = v.q;
    c.k.dm[j] = mont ? v.qinv : v.r[0];
    c.k.dsw[j] = v.r[1];
    c.k.dr2[j] = v.r[2];
    c.k.dr3[j] = v.r[3];
  }
  return mont ? launch_bconv_tcc_any<false, RED_MONTGOMERY>(c, smc, cpsm, st)
              : launch_bconv_tcc_any<false, RED_BAT_LAZY>(c, smc, cpsm, st);
}

int bconv_run(const cross_bconv_plan_s* P, bool bat, const uint32_t* in, int64_t in_ps, int64_t in_ls,
              int64_t in_ts, uint32_t* out, int64_t out_ps, int64_t out_ls, int64_t out_ts, int64_t polys,
              int64_t n, cudaStream_t st, const uint32_t* twist, const uint16_t* trow, const int* trow_host) {
  if (polys == 0 || n == 0) return CROSS_OK;
  if (P->red != CROSS_REDUCTION_BARRETT) {
    set_error("bconv: the HE chains take Barrett plans only (plan reduction %d)", P->red);
    return CROSS_ERR_INVALID_ARG;
  }
  if (bat && P->tc_bimg && in_ts == 1 && out_ts == 1 && n % BT_ROWS == 0 && polys * (n / BT_ROWS) < (1ll << 31)) {
    BconvTcArgs a{in, in_ps, in_ls, out, out_ps, out_ls, (int)polys, (int)n, P->sq, P->sp, P->tc_kb, P->tc_nn, 0,
                  P->src, P->dst, P->qhat_inv, P->tc_bimg, twist, trow, P->err, P->tc_src_fast != 0};
    a.tmem_cols = 64;   // at most 8 CTAs per SM
    while ((int)a.tmem_cols < a.nn) a.tmem_cols <<= 1;
    const int sm_bytes = device_smem_per_sm();
    int ctas = 0;
    const size_t sm = bconv_tc_smem(P->sq, P->sp, P->tc_kb, P->tc_nn, a.tmem_cols, (size_t)sm_bytes, &ctas);
    static const bool generic_only = getenv("CROSS_B200_BCONV_GENERIC") && getenv("CROSS_B200_BCONV_GENERIC")[0] == '1';
    if (sm && P->tc_fast && P->tc_src_fast && (!twist || trow_host) && !generic_only) {
      // targets [j0, j1) from image bimg of MMA width nn
      auto run = [&](int j0, int j1, const uint8_t* bimg, int nn) -> int {
        BconvTccArgs c{in, in_ps, in_ls, out + (int64_t)j0 * out_ls, out_ps, out_ls, (int)polys, (int)n, P->sq,
                       j1 - j0, P->tc_kb, nn, 64, bimg, P->err, {}};
        while ((int)c.tmem_cols < nn) c.tmem_cols <<= 1;
        int cpsm = 0;
        const size_t smc = bconv_tc_smem(P->sq, j1 - j0, P->tc_kb, nn, c.tmem_cols, (size_t)sm_bytes, &cpsm);
        if (!smc) {
          set_error("bconv: no shared-memory split for size_p=%d", j1 - j0);
          return CROSS_ERR_UNSUPPORTED;
        }
        for (int i = 0; i < P->sq; ++i) {
          const ModC& mc = P->src_host[i];
          c.k.sq_q[i] = (uint32_t)mc.q;
          c.k.sq_m[i] = (uint32_t)mc.m;
          c.k.sq_sw[i] = mc.s_w;
          c.k.sq_hi[i] = P->qhat_inv_host[i];
        }
        for (int j = j0; j < j1; ++j) {
          const ModC& mc = P->dst_host[j];
          c.k.dq[j - j0] = (uint32_t)mc.q;
          c.k.dm[j - j0] = (uint32_t)mc.m;
          c.k.dsw[j - j0] = mc.s_w;
          c.k.tp[j - j0] = twist ? twist + (int64_t)trow_host[j] * n : nullptr;
        }
        return twist ? launch_bconv_tcc_any<true>(c, smc, cpsm, st) : launch_bconv_tcc_any<false>(c, smc, cpsm, st);
      };
      return run(0, P->sp, P->tc_bimg, P->tc_nn);
    }
    if (sm) {
      const bool f = P->tc_fast != 0;
      if (twist)
        return f ? launch_bconv_tc_any<true, true>(a, sm, ctas, st) : launch_bconv_tc_any<false, true>(a, sm, ctas, st);
      return f ? launch_bconv_tc_any<true, false>(a, sm, ctas, st) : launch_bconv_tc_any<false, false>(a, sm, ctas, st);
    }
  }
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

int cross_bconv_plan_create_ex(cross_moduli src, cross_moduli dst, int reduction, const uint32_t* qhat_inv_modq,
                               const uint32_t* qhat_inv_modq_shoup, const uint32_t* qhat_modp,
                               const uint32_t* qhat_modp_shoup, const uint8_t* qhat_modp_bat,
                               cross_bconv_plan* out) {
  CROSS_REQUIRE(src && dst && qhat_inv_modq && qhat_modp && qhat_modp_bat && out,
                "cross_bconv_plan_create: null argument");
  CROSS_REQUIRE(reduction >= CROSS_REDUCTION_BARRETT && reduction <= CROSS_REDUCTION_BAT_LAZY,
                "cross_bconv_plan_create_ex: unknown reduction %d", reduction);
  CROSS_REQUIRE(reduction != CROSS_REDUCTION_SHOUP || (qhat_inv_modq_shoup && qhat_modp_shoup),
                "cross_bconv_plan_create_ex: Shoup plans need the companion tables");
  *out = nullptr;
  auto* P = new cross_bconv_plan_s();
  P->red = reduction;
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
  P->qhat_inv_host = qi;
  // tensor-core B operand: row n = 4j + b, K byte 4i + a, in the K-major
  // no-swizzle core-matrix layout of k_bconv_tc (sq <= 32, sp <= 64)
  std::vector<uint8_t> bimg;
  // the tensor-core image serves every reduction whose basis_change_bat is a
  // BAT contraction (Barrett, Montgomery, BAT-lazy; not Shoup, bconv.py:244)
  if (reduction != CROSS_REDUCTION_SHOUP && sq <= 32 && sp <= 64) {
    P->tc_kb = (sq + 7) / 8;
    P->tc_nn = (4 * sp + 15) / 16 * 16;
    const int kb = P->tc_kb;
    // image of the targets [j0, j1): row n = 4 (j - j0) + b, K byte 4i + a
    auto image = [&](int j0, int j1, std::vector<uint8_t>& img) {
      const int nn = (4 * (j1 - j0) + 15) / 16 * 16;
      img.assign((size_t)kb * (nn / 8) * 256, 0);
      for (int n = 0; n < 4 * (j1 - j0); ++n)
        for (int i = 0; i < sq; ++i) {
          const uint32_t word = bat[((size_t)4 * j0 + n) * sq + i];   // bat[j][b][i], row 4j + b
          for (int a = 0; a < 4; ++a) {
            const int kbyte = 4 * i + a, k = kbyte / 32, kk = kbyte % 32;
            img[(size_t)k * (nn / 8) * 256 + (n / 8) * 256 + (kk / 16) * 128 + (n % 8) * 16 + kk % 16] =
                (uint8_t)(word >> (8 * a));
          }
        }
      return nn;
    };
    image(0, sp, bimg);
    bool fast = true;
    for (const ModC& mc : P->dst_host) fast = fast && reduce_fast_ok(mc);
    for (const ModC& mc : P->src_host) fast = fast && barrett_w32_ok(mc);
    P->tc_fast = fast ? 1 : 0;
    bool src_fast = true;
    for (const ModC& mc : P->src_host) src_fast = src_fast && reduce_fast_ok(mc);
    P->tc_src_fast = src_fast ? 1 : 0;
  }
  std::vector<int> zero(1, 0);
  int rc = upload_vec(&P->src, P->src_host);
  if (!rc) rc = upload(&P->err, zero.data(), 1);
  if (!rc && !bimg.empty() && !(getenv("CROSS_B200_DISABLE_TC") && getenv("CROSS_B200_DISABLE_TC")[0] == '1')) {
    rc = upload_vec(&P->tc_bimg, bimg);
  }
  if (!rc) rc = upload_vec(&P->dst, P->dst_host);
  if (!rc) rc = upload_vec(&P->qhat_inv, qi);
  if (!rc) rc = upload_vec(&P->bat, bat);
  if (!rc) rc = upload_vec(&P->qhat_modp, qm);
  if (!rc && reduction != CROSS_REDUCTION_BARRETT) {
    P->src_v_host = make_varc(P->src_host);
    P->dst_v_host = make_varc(P->dst_host);
    rc = upload_vec(&P->src_v, P->src_v_host);
    if (!rc) rc = upload_vec(&P->dst_v, P->dst_v_host);
    if (!rc && reduction == CROSS_REDUCTION_SHOUP) {
      std::vector<uint32_t> qs(qhat_inv_modq_shoup, qhat_inv_modq_shoup + sq), qms((size_t)sp * sq);
      for (int i = 0; i < sq; ++i)
        for (int j = 0; j < sp; ++j) qms[(size_t)j * sq + i] = qhat_modp_shoup[(size_t)i * sp + j];
      rc = upload_vec(&P->qhat_inv_s, qs);
      if (!rc) rc = upload_vec(&P->qhat_modp_s, qms);
    }
  }
  if (rc) {
    cross_bconv_plan_destroy(P);
    return rc;
  }
  *out = P;
  return CROSS_OK;
}

int cross_bconv_plan_create(cross_moduli src, cross_moduli dst, const uint32_t* qhat_inv_modq,
                            const uint32_t* qhat_modp, const uint8_t* qhat_modp_bat, cross_bconv_plan* out) {
  return cross_bconv_plan_create_ex(src, dst, CROSS_REDUCTION_BARRETT, qhat_inv_modq, nullptr, qhat_modp, nullptr,
                                    qhat_modp_bat, out);
}

int cross_bconv_output_bytes(cross_bconv_plan P) {
  CROSS_REQUIRE(P, "cross_bconv_output_bytes: null plan");
  return P->red == CROSS_REDUCTION_BAT_LAZY ? 8 : 4;
}

int cross_bconv_plan_destroy(cross_bconv_plan P) {
  if (!P) return CROSS_OK;
  dfree(P->src);
  dfree(P->dst);
  dfree(P->qhat_inv);
  dfree(P->bat);
  dfree(P->qhat_modp);
  dfree(P->tc_bimg);
  dfree(P->err);
  dfree(P->src_v);
  dfree(P->dst_v);
  dfree(P->qhat_inv_s);
  dfree(P->qhat_modp_s);
  delete P;
  return CROSS_OK;
}

int cross_bconv_plan_check(cross_bconv_plan P) {
  CROSS_REQUIRE(P, "cross_bconv_plan_check: null plan");
  int e = 0;
  CROSS_CHECK_CUDA(cudaMemcpy(&e, P->err, sizeof(int), cudaMemcpyDeviceToHost));
  if (e) {
    const int zero = 0;
    CROSS_CHECK_CUDA(cudaMemcpy(P->err, &zero, sizeof(int), cudaMemcpyHostToDevice));
    set_error("tensor-core basis conversion: a bounded wait expired (code %d); output invalid", e);
    return CROSS_ERR_TIMEOUT;
  }
  return CROSS_OK;
}

int cross_bconv_ex(cross_bconv_plan P, int bat, const uint32_t* in, void* out, int64_t batch, int64_t n,
                   int layout, void* stream) {
  CROSS_REQUIRE(P && batch >= 0 && n >= 0 && (batch == 0 || n == 0 || (in && out && (const void*)in != out)),
                "cross_bconv_ex: bad argument");
  if (P->red == CROSS_REDUCTION_BARRETT) return cross_bconv(P, bat, in, (uint32_t*)out, batch, n, layout, stream);
  const int sq = P->sq, sp = P->sp;
  if (layout == CROSS_LAYOUT_REFERENCE)
    return bconv_var_run(P, bat != 0, in, n * sq, 1, sq, out, n * sp, 1, sp, batch, n, (cudaStream_t)stream);
  CROSS_REQUIRE(layout == CROSS_LAYOUT_LIMB_MAJOR, "cross_bconv_ex: unknown layout %d", layout);
  return bconv_var_run(P, bat != 0, in, n * sq, n, 1, out, n * sp, n, 1, batch, n, (cudaStream_t)stream);
}

int cross_bconv(cross_bconv_plan P, int bat, const uint32_t* in, uint32_t* out, int64_t batch, int64_t n,
                int layout, void* stream) {
  CROSS_REQUIRE(P && batch >= 0 && n >= 0 && (batch == 0 || n == 0 || (in && out && in != out)),
                "cross_bconv: bad argument");
  CROSS_REQUIRE(P->red != CROSS_REDUCTION_BAT_LAZY,
                "cross_bconv: BAT-lazy plans produce uint64 outputs; use cross_bconv_ex");
  if (P->red != CROSS_REDUCTION_BARRETT) return cross_bconv_ex(P, bat, in, out, batch, n, layout, stream);
  const int sq = P->sq, sp = P->sp;
  if (layout == CROSS_LAYOUT_REFERENCE)
    return bconv_run(P, bat != 0, in, n * sq, 1, sq, out, n * sp, 1, sp, batch, n, (cudaStream_t)stream);
  CROSS_REQUIRE(layout == CROSS_LAYOUT_LIMB_MAJOR, "cross_bconv: unknown layout %d", layout);
  return bconv_run(P, bat != 0, in, n * sq, n, 1, out, n * sp, n, 1, batch, n, (cudaStream_t)stream);
}

}  // extern "C"
