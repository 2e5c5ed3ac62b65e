// Internal plan structures and launchers shared by the translation units.
#pragma once

#include <cuda.h>

#include <atomic>
#include <cstdint>
#include <vector>

#include "common.cuh"

struct cross_moduli_s {
  int n = 0;
  std::vector<cross::ModC> host;
  cross::ModC* dev = nullptr;
  cross::VarC* dev_v = nullptr;     // Montgomery / Shoup / BAT-lazy constants of the same moduli
  uint4* dev_f = nullptr;           // per modulus {q, m, s_w, forms}: the element-wise kernels' packed
                                    // Barrett constants (forms bit 0: barrett_w32 exact, bit 1: reduce_fast exact)
};

// NTT plan: the reference's BAT tables re-laid out for the kernels.
// "col" matrices contract over the row index r of the (r, c) matrix
// (ntt step 1 "brcmq,zqrpm", intt step 3 "brcmq,lqrpm"); "row" matrices
// contract over the column index (ntt step 3 "brcmq,cqnpm", intt step 1
// "brcmq,cqlpm").
struct cross_ntt_plan_s {
  int r = 0, c = 0, M = 0;
  int red = CROSS_REDUCTION_BARRETT;   // cross_reduction of the transform's reductions
  std::vector<cross::ModC> mods_host;
  cross::ModC* mods = nullptr;      // [M]
  cross::VarC* varc = nullptr;      // [M] Montgomery / BAT-lazy constants (variant plans)
  // Shoup plans (CUDA-core path): plain uint32 tables and their companions
  // floor(T 2^32 / q), per limb, row-major:
  //   sh[0] ntt T1 [M][r][r]   sh[1] ntt T2 [M][r][c]   sh[2] ntt T3 [M][c][c]
  //   sh[3] intt T1 [M][c][c]  sh[4] intt T2 [M][r][c]  sh[5] intt T3 [M][r][r]
  uint32_t* sh[6] = {};
  uint32_t* sh_s[6] = {};
  // dp4a operands: 4 bytes over q packed into one u32, planes p separate.
  uint32_t* col_fwd = nullptr;      // [M][4 p][r z][r k]   from ntt_bat_tf_step1
  uint32_t* col_inv = nullptr;      // [M][4 p][r l][r k]   from intt_bat_tf_step3
  uint32_t* row_fwd = nullptr;      // [M][4 p][c k][c n]   from ntt_bat_tf_step3
  uint32_t* row_inv = nullptr;      // [M][4 p][c k][c n]   from intt_bat_tf_step1
  uint32_t* tw_fwd = nullptr;       // [M][r][c]            ntt_tf_step2
  uint32_t* tw_inv = nullptr;       // [M][r][c]            intt_tf_step2
  uint16_t* identity = nullptr;     // [M] 0..M-1
  // tcgen05 operands (r and c multiples of 128): B matrices (4*nout x 4*kw bytes
  // per limb, row 4n + p, column 4w + q) with their TMA descriptors.
  bool tc = false;
  uint8_t* tc_col_fwd = nullptr;    // [M][4r][4r]  from ntt_bat_tf_step1
  uint8_t* tc_col_inv = nullptr;    // [M][4r][4r]  from intt_bat_tf_step3
  uint8_t* tc_row_fwd = nullptr;    // [M][4c][4c]  from ntt_bat_tf_step3
  uint8_t* tc_row_inv = nullptr;    // [M][4c][4c]  from intt_bat_tf_step1
  uint32_t* tc_tw_inv = nullptr;    // [M][c][r]    intt_tf_step2 transposed
  int* tc_err = nullptr;            // device error word of the tensor-core kernels
  int tc_fast = 0;                  // 32-bit remainder Barrett is exact for every limb
  int tc_pair = 0;                  // two-SM kernel (k_bat_tc2) for K extents kw <= 256
  bool tc64 = false;                // 64 x 64 Barrett plan: plain transforms by k_ntt64 (one launch)
  CUtensorMap tm_col_fwd, tm_col_inv, tm_row_fwd, tm_row_inv;       // boxes of 256 B rows
  CUtensorMap tm2_col_fwd, tm2_col_inv, tm2_row_fwd, tm2_row_inv;   // boxes of 128 B rows
};

struct cross_bconv_plan_s {
  int sq = 0, sp = 0;
  int red = CROSS_REDUCTION_BARRETT;   // cross_reduction of the source / target contexts
  cross::VarC* src_v = nullptr;        // [sq] variant constants of the source moduli
  cross::VarC* dst_v = nullptr;        // [sp] variant constants of the target moduli
  std::vector<cross::VarC> src_v_host, dst_v_host;
  uint32_t* qhat_inv_s = nullptr;      // [sq]      Shoup companion of qhat_inv
  uint32_t* qhat_modp_s = nullptr;     // [sp][sq]  Shoup companion of qhat_modp
  int tc_fast = 0;                  // tensor-core kernel may use reduce_fast / barrett_w32
  int tc_src_fast = 0;              // reduce_fast is exact for every source modulus
  int tc_kb = 0, tc_nn = 0;         // K blocks of 8 source limbs, MMA N (4 sp rounded up to 16)
  uint8_t* tc_bimg = nullptr;       // B operand in its shared-memory image (K-major, no swizzle)
  int* err = nullptr;               // device error word of the tensor-core kernel
  std::vector<cross::ModC> src_host, dst_host;
  cross::ModC* src = nullptr;       // [sq]
  cross::ModC* dst = nullptr;       // [sp]
  uint32_t* qhat_inv = nullptr;     // [sq]
  std::vector<uint32_t> qhat_inv_host;   // [sq] (the constant-bank kernel's parameters)
  uint32_t* bat = nullptr;          // [sp][4 b][sq]: sum_a bat[(i*4+a), j, b] << 8a
  uint32_t* qhat_modp = nullptr;    // [sp][sq]
};

namespace cross {

// A positive int cached per CUDA device (0 = not computed yet); safe to read and
// fill from several host threads (a racing first use computes the same value).
struct PerDevice {
  static constexpr int kDevices = 64;
  std::atomic<int> v[kDevices];
  template <class F>
  int get(F&& compute) {
    int d = 0;
    if (cudaGetDevice(&d) != cudaSuccess || d < 0 || d >= kDevices) return compute();
    int x = v[d].load(std::memory_order_relaxed);
    if (x <= 0) {
      x = compute();
      v[d].store(x, std::memory_order_relaxed);
    }
    return x;
  }
};
// Multiprocessors and shared memory per multiprocessor of the current device.
int device_sm_count();
int device_smem_per_sm();

// reduce_fast (tc_ptx.cuh) returns finite_field.py's Barrett value exactly for
// modulus mc when the true remainder z - t q stays inside (-(2^32 - q), 2^32)
// for every input: with t = floor(z m / 2^s) and m within one of 2^s / q,
// |r| < (z / 2^s + 2) q, checked here for z < 2^53 and z < 2^31 q + 2^32 (a
// product of a word below 2^31 and a residue, plus a word).
inline bool reduce_fast_ok(const ModC& mc) {
  if (mc.w != 32 || mc.s_w >= 32 || mc.m >= (1ull << 32)) return false;
  const unsigned __int128 q = mc.q;
  const unsigned s_bits = mc.w + mc.s_w;
  const unsigned __int128 lim = ((unsigned __int128)1 << 32) - q;
  for (unsigned __int128 z : {(unsigned __int128)1 << 53, ((unsigned __int128)1 << 31) * q + ((unsigned __int128)1 << 32)})
    if (((z >> s_bits) + 3) * q >= lim) return false;
  return true;
}
// barrett_w32 (common.cuh) equals barrett for this modulus.
inline bool barrett_w32_ok(const ModC& mc) { return mc.w == 32 && mc.m < (1ull << 32); }

// Reduction applied by a contraction epilogue (template argument of the
// kernels): the reference Barrett (generic or the exact 32-bit forms), or the
// Montgomery / BAT-lazy variants of the NTT.
enum RedMode { RED_BARRETT = 0, RED_BARRETT_FAST = 1, RED_MONTGOMERY = 2, RED_BAT_LAZY = 3 };

// VarC of odd moduli q < 2^31 (cross_moduli guarantees both).
std::vector<VarC> make_varc(const std::vector<ModC>& mods);

// Bump allocator over a caller-provided workspace (or a size query when
// base == nullptr).
struct Arena {
  char* base;
  size_t cap;
  size_t off = 0;
  Arena(void* b, size_t c) : base((char*)b), cap(c) {}
  template <class T>
  T* take(size_t count) {
    size_t bytes = (count * sizeof(T) + 255) & ~(size_t)255;
    T* r = base ? (T*)(base + off) : nullptr;
    off += bytes;
    return r;
  }
  bool ok() const { return base == nullptr || off <= cap; }
};

// A strided set of limb-polynomials: element (poly, slot, t) lives at
// ptr + poly*ps + slot*ss + t.
struct LP {
  const uint32_t* p;
  int64_t ps, ss;
};
struct LPo {
  uint32_t* p;
  int64_t ps, ss;
};

template <class T>
int upload(T** dst, const T* src, size_t count);
template <class T>
int upload_vec(T** dst, const std::vector<T>& v) { return upload(dst, v.data(), v.size()); }
void dfree(void* p);

// Scratch words ntt_run / ntt_exec need for lps limb-polynomials.
int64_t ntt_tmp_words(const cross_ntt_plan_s* plan, int64_t lps);

// Coefficient-domain order of a limb-polynomial: natural (index r*C + c at
// position r*C + c) or transposed (index r*C + c at position c*R + r).  The
// evaluation domain is always in the reference's (bit-reversed) order.
enum CoefLayout { COEF_NATURAL = 0, COEF_TRANSPOSED = 1 };

// An operand that shares the output's position layout.  Element index e of a
// batch splits as (e / E, e % E) with strides (ps, es); slots stride ss.
struct View {
  const uint32_t* p = nullptr;
  int64_t ps = 0, es = 0, ss = 0;
  int E = 1;
  __host__ __device__ const uint32_t* at(int64_t e, int slot) const {
    if (E == 1) return p + e * ps + slot * ss;
    const unsigned c = (unsigned)e / (unsigned)E;   // element indices stay below 2^31
    return p + (int64_t)c * ps + (int64_t)((unsigned)e - c * E) * es + slot * ss;
  }
};

// Position-wise operation fused into the last stage of a transform; r is the
// Barrett-reduced transform output at a position:
//   EPI_MUL      r = Barrett(r * tab[trow[slot]][pos])              (psi twists)
//   EPI_COMBINE  r = Barrett(x[pos] * scal[slot] + r)               (rescale, ciphertext.py:299-302)
//   EPI_MODDOWN  s = x[pos] < r ? x[pos] + q - r : x[pos] - r       (ModDown, hemul.py:198-215)
//                t = Barrett(s * scal[slot]);
//                r = base on for e % E ? (base[pos] + t >= q ? base[pos] + t - q : base[pos] + t) : t
enum EpiOp { EPI_NONE = 0, EPI_MUL = 1, EPI_COMBINE = 2, EPI_MODDOWN = 3 };
struct Epi {
  int op = EPI_NONE;
  const uint32_t* tab = nullptr;
  const uint16_t* trow = nullptr;
  View x;
  const uint32_t* scal = nullptr;
  View base;
  unsigned base_mask = 0;
};

// NTT (inverse = false): input coefficients in `in_layout`, output evaluations.
// INTT (inverse = true): input evaluations, output coefficients in `out_layout`.
// epi is applied to the final output.  tmp holds ntt_tmp_words() words.
int ntt_exec(const cross_ntt_plan_s* plan, bool inverse, LP in, int in_layout, LPo out, int out_layout,
             int64_t polys, int slots, const uint16_t* limbs, const Epi& epi, uint32_t* tmp, cudaStream_t st);

// tensor-core path (ntt_tc.cu)
bool tc_supported(int r, int c);
int tc_plan_init(cross_ntt_plan_s* P, const uint8_t* ntt1, const uint8_t* ntt3, const uint8_t* intt1,
                 const uint8_t* intt3, const uint32_t* intt_tw);
void tc_plan_free(cross_ntt_plan_s* P);
// Plain NTT / INTT of a 64 x 64 plan (tc64), natural coefficient order, one
// launch; in / out limb-polynomial bases and strides 16-byte aligned.
int ntt64_run(const cross_ntt_plan_s* P, bool inverse, LP in, LPo out, int64_t polys, int slots,
              const uint16_t* limbs, cudaStream_t st);
int ntt_exec_tc(const cross_ntt_plan_s* P, bool inverse, LP in, int in_layout, LPo out, int out_layout,
                int64_t polys, int slots, const uint16_t* limbs, const Epi& epi, uint32_t* tmp, cudaStream_t st);

// Natural-order NTT / INTT of a Shoup plan on the CUDA cores (ntt_shoup.cu).
int ntt_run_shoup(const cross_ntt_plan_s* P, bool inverse, LP in, LPo out, int64_t polys, int slots,
                  const uint16_t* limbs, uint32_t* tmp, cudaStream_t st);

// basis_change_bat of a Montgomery / BAT-lazy plan on the tensor cores
// (bconv.cu); CROSS_ERR_UNSUPPORTED, nothing launched, for shapes it does not
// take (strided coefficients, n % 128 != 0).
int bconv_var_tc(const cross_bconv_plan_s* P, const uint32_t* in, int64_t in_ps, int64_t in_ls, int64_t in_ts,
                 void* out, int64_t out_ps, int64_t out_ls, int64_t out_ts, int64_t polys, int64_t n,
                 cudaStream_t st);
// Basis conversion of a Montgomery / Shoup / BAT-lazy plan (bconv_var.cu);
// out is uint64 for BAT-lazy plans, else uint32 (strides in elements).
int bconv_var_run(const cross_bconv_plan_s* P, bool bat, const uint32_t* in, int64_t in_ps, int64_t in_ls,
                  int64_t in_ts, void* out, int64_t out_ps, int64_t out_ls, int64_t out_ts, int64_t polys,
                  int64_t n, cudaStream_t st);

// NTT over polys x slots limb-polynomials (internal layout); limbs[slot] is the
// plan limb of each slot (device array).  tmp holds ntt_tmp_words() words.
int ntt_run(const cross_ntt_plan_s* plan, bool inverse, LP in, LPo out, int64_t polys, int slots,
            const uint16_t* limbs, uint32_t* tmp, cudaStream_t st);

// bconv over polys with arbitrary limb / coefficient strides.  With tab set,
// output limb j is further multiplied by tab[trow[j]][t] (position t) and
// Barrett-reduced with the target modulus (the psi twist of ciphertext.py:496).
// trow_host: the same rows on the host (lets the tensor-core kernel take the
// twist rows as parameters; without it a twisted conversion takes the
// generic kernel).
int bconv_run(const cross_bconv_plan_s* plan, bool bat, const uint32_t* in, int64_t in_ps,
              int64_t in_ls, int64_t in_ts, uint32_t* out, int64_t out_ps, int64_t out_ls,
              int64_t out_ts, int64_t polys, int64_t n, cudaStream_t st, const uint32_t* tab = nullptr,
              const uint16_t* trow = nullptr, const int* trow_host = nullptr);

// y[poly, slot, t] = Barrett_{mods[midx[slot]]}(x * tab[trow[slot] * n + t])
int modmul_table_lm(LP x, LPo y, int64_t polys, int slots, int64_t n, const uint32_t* tab,
                    const uint16_t* trow, const ModC* mods, const uint16_t* midx, cudaStream_t st);
// Strided batched transpose of limb-polynomials: out[lp][c][r] = in[lp][r][c]
// for (rows x cols) matrices; any sizes.
int transpose_lp(LP in, LPo out, int64_t polys, int slots, int rows, int cols, cudaStream_t st);
// Apply epi (EpiOp) in place to out, N words per limb-polynomial.
int apply_epi(const Epi& e, LPo out, int64_t polys, int slots, int64_t N, const uint16_t* limbs, const ModC* mods,
              cudaStream_t st);
// batched 2-D transpose: in (batch, rows, cols) -> out (batch, cols, rows)
int transpose_u32(const uint32_t* in, uint32_t* out, int64_t batch, int64_t rows, int64_t cols,
                  cudaStream_t st);

}  // namespace cross
