/*
 * cross_b200.h -- C ABI of the B200-native (sm_100a) CKKS hot path of
 * EfficientPPML/CROSS (jaxite_word).
 *
 * Conventions
 *   - Every entry point returns 0 (CROSS_OK) or a negative cross_status;
 *     nothing is thrown across the ABI.  cross_last_error() returns a
 *     per-thread message describing the last failure.
 *   - Device buffers are caller-owned.  Operators that need scratch take a
 *     (workspace, workspace_bytes) pair sized by the matching
 *     *_workspace_size() query; nothing is allocated on the operator path.
 *     Plan creation allocates and uploads the plan's constants once.
 *   - `stream` is a cudaStream_t passed as void* (NULL = legacy stream).
 *   - Plans are immutable after creation (the *_set_keys calls complete
 *     creation) and may be used concurrently on different streams.
 *   - Integer semantics are those of the reference: uint32 residues, uint64
 *     intermediates with wrap-around, lazy Barrett outputs (values may lie in
 *     [q, 2q)), so results are bit-identical to jaxite_word.
 *   - Layouts: CROSS_LAYOUT_REFERENCE is jaxite_word's (..., r, c, limbs),
 *     limb-innermost.  CROSS_LAYOUT_LIMB_MAJOR is (..., limbs, r, c): each
 *     limb-polynomial contiguous, the internal layout of the kernels.
 *     CROSS_LAYOUT_LIMB_MAJOR_TRANSPOSED (cross_ntt only) is limb-major with
 *     the coefficient side in transposed order (coefficient r*C + c stored at
 *     c*R + r), the order the tensor-core transforms work in: an NTT from it
 *     and an INTT into it skip a transpose pass.
 */
#ifndef CROSS_B200_H_
#define CROSS_B200_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define CROSS_B200_ABI_VERSION 1

typedef enum cross_status {
  CROSS_OK = 0,
  CROSS_ERR_INVALID_ARG = -1,
  CROSS_ERR_CUDA = -2,
  CROSS_ERR_UNSUPPORTED = -3,
  CROSS_ERR_WORKSPACE = -4,
  CROSS_ERR_TIMEOUT = -5
} cross_status;

typedef enum cross_layout {
  CROSS_LAYOUT_REFERENCE = 0,
  CROSS_LAYOUT_LIMB_MAJOR = 1,
  CROSS_LAYOUT_LIMB_MAJOR_TRANSPOSED = 2
} cross_layout;

/* Modular reduction of a transform or basis conversion: the finite_field.py
 * context the reference builds it on. */
typedef enum cross_reduction {
  CROSS_REDUCTION_BARRETT = 0,      /* BarrettContext    (finite_field.py:170-272) */
  CROSS_REDUCTION_MONTGOMERY = 1,   /* MontgomeryContext (finite_field.py:58-164)  */
  CROSS_REDUCTION_SHOUP = 2,        /* ShoupContext      (finite_field.py:278-338) */
  CROSS_REDUCTION_BAT_LAZY = 3      /* BATLazyContext    (finite_field.py:344-428) */
} cross_reduction;

typedef struct cross_moduli_s* cross_moduli;
typedef struct cross_ntt_plan_s* cross_ntt_plan;
typedef struct cross_bconv_plan_s* cross_bconv_plan;
typedef struct cross_hemul_plan_s* cross_hemul_plan;
typedef struct cross_herot_plan_s* cross_herot_plan;

int cross_abi_version(void);
const char* cross_last_error(void);
/* Number of CUDA kernels this library has launched in the process (all
 * threads); a diagnostic for benchmarks. */
uint64_t cross_launch_count(void);

/* Throughput probe of the int8 tensor cores (no counterpart in the
 * reference; the measured peak that the contraction kernels' roofline
 * fractions are quoted against).  One launch on all SMs: each CTA issues
 * kchunks x 4 tcgen05.mma kind::i8 of K = 32 bytes on operands resident in
 * shared memory, M = 128 x N = 256 per CTA (pair = 0) or M = 256 x N = 256 per
 * cluster of two CTAs with cta_group::2 (pair != 0, the form of the NTT
 * contraction), i.e. 2 * 128 * 256 * 128 int8 operations per CTA per chunk.
 * *ctas (host) receives the CTAs launched; err is a device int that the
 * bounded completion wait sets to 31 when it expires.  1 <= kchunks <= 2^20. */
int cross_tc_i8_probe(int pair, int64_t kchunks, int* err, int* ctas, void* stream);

/* Self-test of the bounded device waits (no counterpart in the reference):
 * one warp waits, through the same bounded mbarrier wait the tensor-core
 * kernels use, on a barrier that nothing arrives on.  The wait must give up
 * after bound_ns of global timer (1 us .. 1 s), record its code and let the
 * kernel return; the call synchronizes the stream and returns
 * CROSS_ERR_TIMEOUT when that happened as intended (the context stays
 * usable), CROSS_ERR_CUDA otherwise. */
int cross_wait_selftest(uint64_t bound_ns, void* stream);

/* ------------------------------------------------------------------ */
/* Modulus sets                                                        */
/* ------------------------------------------------------------------ */

/* A list of RNS moduli with their Barrett constants.
 * Replaces finite_field.BarrettContext.__init__ (finite_field.py:171-185):
 * barrett_m = floor(2^s / q), barrett_w = min(s, 32),
 * barrett_s_w = s - w with s = 2*ceil(log2 q), computed by the caller.
 * Moduli must be odd and below 2^31 (ntt_mm.py:142).  Host arrays. */
int cross_moduli_create(int num_moduli, const uint32_t* moduli, const uint64_t* barrett_m,
                        const uint32_t* barrett_w, const uint32_t* barrett_s_w,
                        cross_moduli* out);
int cross_moduli_destroy(cross_moduli moduli);

/* ------------------------------------------------------------------ */
/* Elementwise modular kernels (reference layout: last axis = limbs;   */
/* `rows` is the product of all other axes)                            */
/* ------------------------------------------------------------------ */

/* BarrettContext.modular_reduction (finite_field.py:201-230) as used by
 * Ciphertext.mod_reduce (ciphertext.py:195-197): out[i,m] = Barrett_m(in[i,m]).
 * `in` is uint64 when in_is_u64, else uint32. */
int cross_mod_reduce(cross_moduli moduli, const void* in, int in_is_u64, uint32_t* out,
                     int64_t rows, void* stream);

/* MontgomeryContext / ShoupContext / BATLazyContext.modular_reduction
 * (finite_field.py:94-154, 305-330, 384-425), moduli on the last axis:
 * z (rows, M) uint64 and, for Shoup, its companion product z_s (rows, M);
 * out (rows, M) uint32, or uint64 for CROSS_REDUCTION_BAT_LAZY.
 * CROSS_REDUCTION_BARRETT is cross_mod_reduce of uint64 input. */
int cross_mod_reduce_ex(cross_moduli moduli, int reduction, const uint64_t* z, const uint64_t* z_s, void* out,
                        int64_t rows, void* stream);

/* Ciphertext.modmul (ciphertext.py:189-193) with the broadcast the reference
 * uses for its constant tables: out[i,m] = Barrett_m(a[i,m] * b[i % b_rows, m])
 * computed in uint64 with wrap-around. */
int cross_modmul(cross_moduli moduli, const void* a, int a_is_u64, const void* b, int b_is_u64,
                 int64_t b_rows, uint32_t* out, int64_t rows, void* stream);

/* Ciphertext.ciphertext_mult (ciphertext.py:309-324).  ct: (batch, 4, n, M);
 * out01: (batch, 2, n, M) = (a0*b0, a0*b1 + a1*b0); out2: (batch, 1, n, M) = a1*b1. */
int cross_tensor_product(cross_moduli moduli, const uint32_t* ct, uint32_t* out01, uint32_t* out2,
                         int64_t batch, int64_t n, void* stream);

/* The key-switch inner product of Ciphertext.key_switch (ciphertext.py:506-518,
 * herot.py:236-246): ext[j] (j < dnum <= 16; a host array of device pointers) is
 * digit j's extended ciphertext in restored limb order, (batch, n, M) for
 * CROSS_LAYOUT_REFERENCE or (batch, M, n) for CROSS_LAYOUT_LIMB_MAJOR; evk_a,
 * evk_b are the key's limbs in the same order, (dnum, n, M) or (dnum, M, n);
 * out (batch, 2, n, M) or (batch, 2, M, n):
 *   out[:, 0] = Barrett(sum_j ext[j] evk_b[j]),  out[:, 1] = Barrett(sum_j ext[j] evk_a[j]),
 * the sums in uint64 with wrap-around.  moduli: the M limbs (Q' then P). */
int cross_ks_inner_product(cross_moduli moduli, const uint32_t* const* ext, int dnum, const uint32_t* evk_a,
                           const uint32_t* evk_b, uint32_t* out, int64_t batch, int64_t n, int layout, void* stream);

/* The ModDown tail of hemul.py:199-207 and 214-215 (herot.py:277-296):
 * x, y, out (rows, M), limbs last; s = x < y ? x + q - y : x - y in uint32,
 * t = Barrett(s * p_inv_mod_q[m]) (p_inv_mod_q: device array of M, P^-1 mod q_m);
 * out = base + t, minus q where that is >= q, when base (rows, M) is not NULL,
 * else t. */
int cross_moddown_sub_mul(cross_moduli moduli, const uint32_t* x, const uint32_t* y, const uint32_t* p_inv_mod_q,
                          const uint32_t* base, uint32_t* out, int64_t rows, void* stream);

/* The centred lift of rescale (ciphertext.py:279-295): last (polys, n) is the
 * coefficient-form last limb (Barrett outputs of modulus q_last); gamma_psi
 * holds gamma_i psi_i^t, (n, M) for CROSS_LAYOUT_REFERENCE or (M, n) for
 * CROSS_LAYOUT_LIMB_MAJOR; out (polys, n, M) or (polys, M, n):
 *   out = Barrett_i((last < (q_last + 1) / 2 ? last : q_i - q_last + last) * gamma_psi)
 * with the lift in uint64.  moduli: the M = L - 1 remaining moduli. */
int cross_rescale_lift(cross_moduli moduli, const uint32_t* last, uint32_t q_last, const uint32_t* gamma_psi,
                       uint32_t* out, int64_t polys, int64_t n, int layout, void* stream);

/* add.jax_add (add.py:7-27): a, b, out (elements, M, n); result a+b (uint32
 * wrap) minus q where it is strictly greater than q. */
int cross_add_mod(cross_moduli moduli, const uint32_t* a, const uint32_t* b, uint32_t* out,
                  int64_t elements, int64_t n, void* stream);

/* Galois automorphism of herot.py:300: out[b, e, j, :] = in[b, e, coef_map[j], :]
 * for in/out (batch*elements, n, M); coef_map is a device int32 array of n. */
int cross_automorphism(const uint32_t* in, const int32_t* coef_map, uint32_t* out,
                       int64_t polys, int64_t n, int num_limbs, void* stream);

/* Layout conversion between (polys, n, M) and (polys, M, n). */
int cross_to_limb_major(const uint32_t* in, uint32_t* out, int64_t polys, int64_t n, int num_limbs,
                        void* stream);
int cross_to_reference(const uint32_t* in, uint32_t* out, int64_t polys, int64_t n, int num_limbs,
                       void* stream);

/* ------------------------------------------------------------------ */
/* BAT matrix NTT / INTT                                               */
/* ------------------------------------------------------------------ */

/* Replaces NTTCiphertextBarrettContext.__init__ (ntt_mm.py:136-181, 421-429):
 * the plan takes the reference's precomputed tables (host arrays, reference
 * shapes) and stores them in the kernels' layouts:
 *   ntt_bat_tf_step1  (r, 4, r, 4, M) u8      ntt_tf_step2  (r, c, M) u32
 *   ntt_bat_tf_step3  (c, 4, c, 4, M) u8
 *   intt_bat_tf_step1 (c, 4, c, 4, M) u8      intt_tf_step2 (r, c, M) u32
 *   intt_bat_tf_step3 (r, 4, r, 4, M) u8
 * (the reference keeps tf_step2 as uint64; every value is below q < 2^31). */
int cross_ntt_plan_create(cross_moduli moduli, int r, int c,
                          const uint8_t* ntt_bat_tf_step1, const uint32_t* ntt_tf_step2,
                          const uint8_t* ntt_bat_tf_step3, const uint8_t* intt_bat_tf_step1,
                          const uint32_t* intt_tf_step2, const uint8_t* intt_bat_tf_step3,
                          cross_ntt_plan* out);
int cross_ntt_plan_destroy(cross_ntt_plan plan);

/* The same transform with another reduction (same table arguments):
 *   CROSS_REDUCTION_BARRETT     cross_ntt_plan_create.
 *   CROSS_REDUCTION_MONTGOMERY  NTTCiphertextMontgomeryContext (ntt_mm.py:432-440)
 *       and ntt_sm.NTTMontgomeryContext (ntt_sm.py:339-346): the tables are
 *       the reference's Montgomery-form ones (ntt_mm.py:172-181), every
 *       reduction is MontgomeryContext.modular_reduction.
 *   CROSS_REDUCTION_BAT_LAZY    NTTCiphertextBATLazyContext (ntt_mm.py:590-658)
 *       and ntt_sm.NTTBATLazyContext (ntt_sm.py:348-412): Barrett tables; the
 *       first reduction of each transform is BATLazyContext.modular_reduction
 *       (a uint64 value), multiplied by the step-2 table in uint64 with
 *       wrap-around and Barrett-reduced; the last reduction is Barrett.
 * `moduli` carries the Barrett constants in every case (the Montgomery and
 * BAT-lazy constants are derived from the moduli). */
int cross_ntt_plan_create_ex(cross_moduli moduli, int r, int c, int reduction,
                             const uint8_t* ntt_bat_tf_step1, const uint32_t* ntt_tf_step2,
                             const uint8_t* ntt_bat_tf_step3, const uint8_t* intt_bat_tf_step1,
                             const uint32_t* intt_tf_step2, const uint8_t* intt_bat_tf_step3,
                             cross_ntt_plan* out);

/* NTTCiphertextShoupContext (ntt_mm.py:443-587) and ntt_sm.NTTShoupContext
 * (ntt_sm.py:415-494): uint32 twiddle tables and their Shoup companions
 * floor(T 2^32 / q), host arrays in the reference shapes, limbs last:
 *   tables[0] ntt_tf_step1 (r, r, M)   tables[1] ntt_tf_step2 (r, c, M)
 *   tables[2] ntt_tf_step3 (c, c, M)   tables[3] intt_tf_step1 (c, c, M)
 *   tables[4] intt_tf_step2 (r, c, M)  tables[5] intt_tf_step3 (r, r, M)
 *   tables[6..11] the *_shoup companions in the same order.
 * Each matrix product is the reference's byte convolution recombined in
 * uint64 (ntt_mm.py:40-65), i.e. the exact sum modulo 2^64, followed by
 * ShoupContext.modular_reduction cast to uint32. */
int cross_ntt_plan_create_shoup(cross_moduli moduli, int r, int c, const uint32_t* const* tables,
                                cross_ntt_plan* out);

/* The plan's cross_reduction. */
int cross_ntt_plan_reduction(cross_ntt_plan plan);

/* Scratch needed by cross_ntt for `batch` polynomials of all plan limbs. */
size_t cross_ntt_workspace_size(cross_ntt_plan plan, int64_t batch, int layout);

/* NTTCiphertextBarrettContext.ntt / .intt (ntt_mm.py:351-407):
 * in/out (batch, r, c, M) for CROSS_LAYOUT_REFERENCE or (batch, M, r, c) for
 * CROSS_LAYOUT_LIMB_MAJOR, uint32.  Output of ntt is in bit-reversed
 * evaluation order, exactly as the reference.  With
 * CROSS_LAYOUT_LIMB_MAJOR_TRANSPOSED the coefficients (ntt input, intt
 * output) are (batch, M, c, r) and the evaluations (batch, M, r, c).
 * in may equal out.  In the limb-major layouts the tensor-core plans read and
 * write in/out in 16-byte pieces: both must be 16-byte aligned, else
 * CROSS_ERR_INVALID_ARG (CROSS_LAYOUT_REFERENCE has no such rule). */
int cross_ntt(cross_ntt_plan plan, int inverse, const uint32_t* in, uint32_t* out, int64_t batch,
              int layout, void* workspace, size_t workspace_bytes, void* stream);

/* Reports (and clears) the error word of the plan's tensor-core kernels:
 * CROSS_OK, or CROSS_ERR_TIMEOUT when a bounded wait inside a kernel expired
 * (the kernel then stopped early and its output is invalid).  Synchronises
 * the device. */
int cross_ntt_plan_check(cross_ntt_plan plan);

/* Allocation-free variant of cross_ntt; it has no counterpart in the
 * reference.  For callers that cannot allocate device memory on their call
 * path (a plugin inside a framework that has already reserved the GPU's
 * memory, a loop that cannot afford cudaFree's synchronisation): it takes
 * only in/out (limb-major layout, (batch, M, r, c) uint32, in may equal out)
 * and keeps the NTT intermediate in a file-scope static device array of
 * CROSS_NTT_NOALLOC_SCRATCH_BYTES per GPU, held until the process exits.
 * The intermediate is two words per input word, so batch * M * r * c must not
 * exceed CROSS_NTT_NOALLOC_MAX_WORDS (CROSS_NTT_NOALLOC_SCRATCH_BYTES / 8 =
 * 2 Mi words, e.g. batch 4 of 8 limbs at N = 2^16), else CROSS_ERR_WORKSPACE
 * before any launch.  It calls no allocator.  The first call on each device
 * looks up the array's device address (cudaGetSymbolAddress) and caches it for
 * the process; make that first call before any stream capture, and do not
 * call cudaDeviceReset afterwards (the cached address would be stale).  All
 * calls share the array: calls that overlap on the GPU (other streams or
 * threads) race, so issue them on one stream. */
#define CROSS_NTT_NOALLOC_SCRATCH_BYTES (16u << 20)
#define CROSS_NTT_NOALLOC_MAX_WORDS (CROSS_NTT_NOALLOC_SCRATCH_BYTES / 8u)
int cross_ntt_noalloc(cross_ntt_plan plan, int inverse, const uint32_t* in, uint32_t* out, int64_t batch,
                      void* stream);

/* ------------------------------------------------------------------ */
/* BAT basis conversion                                                */
/* ------------------------------------------------------------------ */

/* Replaces BConv.control_gen for one (src, dst) control
 * (bconv.py:67-155): qhat_inv_modq (size_q) u32, qhat_modp (size_q, size_p)
 * u32 and its BAT form qhat_modp_bat (4*size_q, size_p, 4) u8. */
int cross_bconv_plan_create(cross_moduli src, cross_moduli dst, const uint32_t* qhat_inv_modq,
                            const uint32_t* qhat_modp, const uint8_t* qhat_modp_bat,
                            cross_bconv_plan* out);
int cross_bconv_plan_destroy(cross_bconv_plan plan);

/* Reports (and clears) the error word of the plan's tensor-core kernel:
 * CROSS_OK, or CROSS_ERR_TIMEOUT when its bounded wait expired (that launch
 * stopped early and its output is invalid).  Synchronises the device. */
int cross_bconv_plan_check(cross_bconv_plan plan);

/* BConv.basis_change_bat (bconv.py:215-252) when bat != 0, else
 * BConv.basis_change (bconv.py:173-212).  CROSS_LAYOUT_REFERENCE:
 * in (batch, n, size_q) -> out (batch, n, size_p);  CROSS_LAYOUT_LIMB_MAJOR:
 * in (batch, size_q, n) -> out (batch, size_p, n). */
int cross_bconv(cross_bconv_plan plan, int bat, const uint32_t* in, uint32_t* out, int64_t batch,
                int64_t n, int layout, void* stream);

/* BConvMontgomery / BConvShoup / BConvBATLazy (bconv.py:261-390), or
 * BConvBarrett for CROSS_REDUCTION_BARRETT (= cross_bconv_plan_create).  The
 * arguments are the control's tables in the context's computation format
 * (bconv.py:67-97): Montgomery form for MONTGOMERY, plain residues otherwise.
 * qhat_inv_modq_shoup (size_q) and qhat_modp_shoup (size_q, size_p) are the
 * Shoup companions of BConvShoup.control_gen (bconv.py:300-314); required for
 * SHOUP, ignored (may be NULL) otherwise. */
int cross_bconv_plan_create_ex(cross_moduli src, cross_moduli dst, int reduction, const uint32_t* qhat_inv_modq,
                               const uint32_t* qhat_inv_modq_shoup, const uint32_t* qhat_modp,
                               const uint32_t* qhat_modp_shoup, const uint8_t* qhat_modp_bat,
                               cross_bconv_plan* out);

/* Bytes per output element of cross_bconv_ex for this plan: 8 for
 * CROSS_REDUCTION_BAT_LAZY (BATLazyContext.modular_reduction returns uint64,
 * finite_field.py:421-425), else 4. */
int cross_bconv_output_bytes(cross_bconv_plan plan);

/* cross_bconv for a plan of any reduction; `out` holds elements of
 * cross_bconv_output_bytes(plan) bytes.  Reference behaviours kept:
 *   - MONTGOMERY basis_change (bat = 0) re-encodes source limb i with target
 *     modulus i (bconv.py:278-280 broadcasts size_q against size_p), so it
 *     needs size_q == size_p or size_p == 1, else CROSS_ERR_INVALID_ARG;
 *   - SHOUP with bat != 0 is CROSS_ERR_UNSUPPORTED (the base-class BAT path
 *     calls the two-operand Shoup reduction with one operand, bconv.py:244). */
int cross_bconv_ex(cross_bconv_plan plan, int bat, const uint32_t* in, void* out, int64_t batch, int64_t n,
                   int layout, void* stream);

/* ------------------------------------------------------------------ */
/* CKKS client side (ckks_ctx.py, key_gen.py)                          */
/* ------------------------------------------------------------------ */
/* Double-precision steps evaluate every complex product as
 * (a.re b.re - a.im b.im, a.re b.im + a.im b.re) and every sum in CPython's
 * order without fused multiply-adds, so with the caller's twiddles (the
 * reference's cmath.exp values) the results are bit-identical. */

/* FFTSpecialInv / FFTSpecial (ckks_ctx.py:48-110) in place on `batch`
 * vectors of nh complex doubles (interleaved re, im); m a power of two, at
 * least 4 nh (decode runs nh = slots with m = 2 degree); roots: the m
 * complex values exp(2 pi i k / m) (_roots), rot: the nh powers of 5 mod m
 * (_rot_group); inv_scale: 1.0 / nh, applied by the inverse transform. */
int cross_fft_special(double* vals, int64_t batch, int nh, int m, const double* roots, const uint32_t* rot,
                      int inverse, double inv_scale, void* stream);

/* max |scale * v| over n doubles, written to *out (device); encode takes
 * ceil(log2) of it (ckks_ctx.py:357-365). */
int cross_ckks_max_abs_scaled(const double* v, int64_t n, double scale, double* out, void* stream);

/* ckks_ctx.py:356-387: the 2 nh coefficients of slot_to_coeffs(y) (y: nh
 * complex doubles) scaled, divided by 2^log_approx, rounded with
 * nearest_int, fitted into every tower (fit_to_native_vector), times
 * 2^log_approx and times factor[t] (device array, NULL = 1) mod q_t:
 * out (M, 2 nh) uint32 coefficients. */
int cross_ckks_quantize(cross_moduli moduli, const double* y, int nh, double scale, int log_approx,
                        const uint32_t* factor, uint32_t* out, void* stream);

/* gen_rns_polynomial (rns.py): signed coefficients x (n) reduced into every
 * tower, non-negative: out (M, n). */
int cross_rns_from_signed(cross_moduli moduli, const int64_t* x, int64_t n, uint32_t* out, void* stream);

/* out[t][i] = x[t][i] * tab[t][i] mod q_t, fully reduced (tab NULL: x mod q_t);
 * x, tab, out (M, n) limb-major. */
int cross_mul_reduce_lm(cross_moduli moduli, const uint32_t* x, const uint32_t* tab, uint32_t* out, int64_t n,
                        void* stream);

/* ckks_decrypt's accumulation (ckks_ctx.py:264-294): c0 + sum_{i>=1} c_i s^i
 * per tower, reduced after every step; c (elements, n, M), s (M, n) in
 * evaluation form; out (M, n). */
int cross_ckks_decrypt_sum(cross_moduli moduli, const uint32_t* c, int elements, const uint32_t* s, uint32_t* out,
                           int64_t n, void* stream);

/* ckks_encrypt's combination (ckks_ctx.py:198-228): c0 = ((v pk0 + ns e0) mod q
 * + m) mod q, c1 = (v pk1 + ns e1) mod q; v, e0, e1, pk0, pk1 (M, n);
 * m, c0, c1 (n, M). */
int cross_ckks_encrypt(cross_moduli moduli, const uint32_t* m, const uint32_t* v, const uint32_t* e0,
                       const uint32_t* e1, const uint32_t* pk0, const uint32_t* pk1, uint64_t noise_scale,
                       uint32_t* c0, uint32_t* c1, int64_t n, void* stream);

/* gen_pke_pair's b (key_gen.py:328-337): ((e ns) mod q - (a s) mod q) mod q, all (M, n). */
int cross_pke_b(cross_moduli moduli, const uint32_t* e, const uint32_t* a, const uint32_t* s, uint64_t noise_scale,
                uint32_t* b, int64_t n, void* stream);

/* modulus_switch (key_gen.py:77-105) of one tower's coefficients v (mod
 * q_from) into every modulus of `to`: the centred value (v, or v - q_from for
 * v >= (q_from + 1) / 2) reduced mod p_t: out (M_to, n). */
int cross_mod_switch_lift(const uint32_t* v, int64_t n, uint32_t q_from, cross_moduli to, uint32_t* out,
                          void* stream);

/* key_switch_gen's b of one part (key_gen.py:228-246): rows i of Q + P,
 * b = (-a s mod q + [P s_old mod q when start <= i < end] + noise_scale e mod q) mod q;
 * a, e, s, b (Q + P, n) evaluations; s_old (Q, n); p_mod_q (Q): P mod q_i. */
int cross_ks_key_b(cross_moduli moduli, const uint32_t* a, const uint32_t* e, const uint32_t* s, const uint32_t* s_old,
                   const uint32_t* p_mod_q, int start, int end, uint64_t noise_scale, uint32_t* b, int64_t n,
                   void* stream);

/* _crt_combine_rns_plaintext (ckks_ctx.py:517-545): rns (n, M) -> out (n,
 * words) little-endian uint32 words of X mod Q.  inv (M): (Q/q_i)^-1 mod q_i;
 * mi (M, words): Q/q_i; q_words (words): Q.  words <= 66, M <= 64. */
int cross_crt_combine(cross_moduli moduli, const uint32_t* rns, int64_t n, const uint32_t* inv, const uint32_t* mi,
                      const uint32_t* q_words, int words, uint32_t* out, void* stream);

/* ckks_decode's first step (ckks_ctx.py:421-441): for slot i < slots, the
 * big-integer coefficients i and i + nh centred at Q/2 (half_words = Q >> 1),
 * converted to double (round to nearest even), times sf_pre, truncated:
 * out (slots) complex doubles.  *overflow (device int) is set when a value
 * does not fit a double (CPython raises OverflowError). */
int cross_ckks_decode_scale(const uint32_t* x, int words, const uint32_t* q_words, const uint32_t* half_words,
                            double sf_pre, int slots, int nh, double* out, int* overflow, void* stream);

/* The approximation-error estimate of ckks_decode (ckks_ctx.py:458-481):
 * *out (device) = the standard deviation (one block, parallel sums). */
int cross_ckks_decode_stddev(const double* cur, int slots, double* out, void* stream);

/* ckks_ctx.py:496-505: out[i] = in[i] scale + conj(in)[i] scale (component-wise). */
int cross_ckks_decode_combine(const double* in, double* out, int slots, double scale, void* stream);

/* ------------------------------------------------------------------ */
/* Rescale by the last prime (ciphertext.py:223-303)                   */
/* ------------------------------------------------------------------ */

typedef struct cross_rescale_plan_s* cross_rescale_plan;

typedef struct cross_rescale_desc {
  int r, c;                   /* degree layout of the ciphertext                        */
  int L;                      /* limbs before rescale                                   */
  cross_ntt_plan ntt_q;       /* plan over Q (L moduli, same order) with (r, c)         */
  const uint32_t* inv_psi_last;  /* (N)      psi_{q_{L-1}}^{-i}     (ciphertext.py:244-248) */
  const uint32_t* gamma_psi;     /* (L-1, N) gamma_i psi_i^i        (ciphertext.py:239-243) */
  const uint32_t* betas;         /* (L-1)    q_{L-1}^{-1} mod q_i   (ciphertext.py:254)     */
} cross_rescale_desc;

/* Ciphertext.modulus_switch_control_gen (ciphertext.py:223-265). */
int cross_rescale_plan_create(const cross_rescale_desc* desc, cross_rescale_plan* out);
int cross_rescale_plan_destroy(cross_rescale_plan plan);
size_t cross_rescale_workspace_size(cross_rescale_plan plan, int64_t polys, int layout);
/* Ciphertext.rescale (ciphertext.py:267-303): in (polys, r, c, L) -> out
 * (polys, r, c, L-1) (limb-major: (polys, L, N) -> (polys, L-1, N)). */
int cross_rescale(cross_rescale_plan plan, const uint32_t* in, uint32_t* out, int64_t polys, int layout,
                  void* workspace, size_t workspace_bytes, void* stream);

/* ------------------------------------------------------------------ */
/* HE-Mult with relinearisation (hemul.py)                             */
/* ------------------------------------------------------------------ */

typedef struct cross_hemul_desc {
  int r, c;            /* HEMul degree layout (hemul.py:12-28)                        */
  int L;               /* limbs of the input ciphertext, |Q| (dropped to L-1 by rescale) */
  int K;               /* special limbs |P|                                           */
  int dnum;            /* key-switch digits (ciphertext.py:354)                       */
  /* plan over Q then P (L + K moduli) with factorisation (r, c)                      */
  cross_ntt_plan ntt_qp;
  /* plan over P with the default factorisation of ciphertext.py:69-70, used by the
   * ModDown INTT (hemul.py:76-77,179-180); may equal ntt_qp when (r, c) is it       */
  cross_ntt_plan ntt_p;
  int ntt_p_limb_offset;   /* index of P[0] inside ntt_p (L when ntt_p == ntt_qp, else 0) */
  /* ceil((L-1)/alpha) controls: digit j -> its complement in Q' + P (bconv indices
   * are positions in the Q' + P list), then one control P -> Q'                    */
  cross_bconv_plan* ks_bconv;
  cross_bconv_plan down_bconv;
  const uint32_t* inv_psi_last;   /* (N)      psi_{q_{L-1}}^{-i}   (hemul.py:47-50)   */
  const uint32_t* gamma_psi;      /* (L-1, N) gamma_i psi_i^i      (ciphertext.py:239-243) */
  const uint32_t* betas;          /* (L-1)                         (ciphertext.py:254) */
  const uint32_t* inv_psi_q;      /* (L-1, N) psi_i^{-i} over Q'   (ciphertext.py:381-394) */
  const uint32_t* psi_qp;         /* (L-1+K, N) psi^i over Q' + P  (ciphertext.py:343-350) */
  const uint32_t* inv_psi_p;      /* (K, N)   psi^{-i} over P      (hemul.py:91-97)    */
  const uint32_t* p_inv_mod_q;    /* (L-1)    P^{-1} mod q_i       (hemul.py:105-111)  */
} cross_hemul_desc;

int cross_hemul_plan_create(const cross_hemul_desc* desc, cross_hemul_plan* out);
/* HEMul.setup_relinearization (hemul.py:134-151, ciphertext.py:445-451):
 * evk_a, evk_b host arrays (dnum, N, key_limbs) with key_limbs >= L-1+K;
 * limbs [0, L-1) and the last K are used. */
int cross_hemul_set_keys(cross_hemul_plan plan, const uint32_t* evk_a, const uint32_t* evk_b,
                         int key_limbs);
int cross_hemul_plan_destroy(cross_hemul_plan plan);
size_t cross_hemul_workspace_size(cross_hemul_plan plan, int64_t batch, int layout);
/* HEMul.mul (hemul.py:153-217): in (batch, 4, r, c, L) -> out (batch, 2, r, c, L-1)
 * (limb-major: (batch, 4, L, r, c) -> (batch, 2, L-1, r, c)). */
int cross_hemul(cross_hemul_plan plan, const uint32_t* in, uint32_t* out, int64_t batch, int layout,
                void* workspace, size_t workspace_bytes, void* stream);

/* ------------------------------------------------------------------ */
/* HE-Mult sharded by RNS limb across GPUs                             */
/* ------------------------------------------------------------------ */
/* The reference shards only the ciphertext batch (util.py:40-58); for large
 * parameter sets each GPU can instead own a contiguous range of the limbs of
 * every ciphertext.  A shard computes exactly cross_hemul's per-limb
 * operations (hemul.py:153-217) for its limbs, so its output limbs are
 * bit-identical to the one-GPU result.  The key switch's two basis
 * conversions need every digit's limbs (ModUp, ciphertext.py:486-498) and
 * every P limb (ModDown, hemul.py:179-186) in coefficient form, which the
 * caller exchanges between the phases (an all-gather over the ranks, e.g.
 * NCCL over NVLink):
 *   1. cross_hemul_shard_modup_input: in (B, 4, nq + 1, N) limb-major, the
 *      owned Q' limbs then the last limb of Q -> cc_out (nq, B, N):
 *      INTT(d2) psi^-i of the owned limbs, coefficient order transposed;
 *   2. all-gather into cc_all, Q' limb l at cc_all + l * B * N;
 *   3. cross_hemul_shard_keyswitch: cc_all -> kp_out (np, 2 B, N): the owned
 *      P limbs of INTT(KS) psi^-i for both elements (e' = 2 b + e);
 *   4. all-gather into kp_all, P limb k at kp_all + k * 2 * B * N;
 *   5. cross_hemul_shard_moddown: kp_all -> out (B, 2, nq, N), limb-major.
 * Q' is Q without its last modulus; nq = q_end - q_begin, np = p_end -
 * p_begin.  The phases share the workspace (cross_hemul_shard_workspace_size)
 * and must run in order on one stream per shard. */
typedef struct cross_hemul_shard_s* cross_hemul_shard;
typedef struct cross_hemul_shard_desc {
  cross_hemul_plan plan;        /* the HE-Mult plan with its keys set          */
  int q_begin, q_end;           /* owned limbs of Q'                            */
  int p_begin, p_end;           /* owned limbs of P                             */
  /* per key-switch digit j: BConv control digit j -> the owned limbs outside
   * digit j (owned Q' limbs, then owned P limbs, in Q' + P order); NULL where a
   * shard has no such limb */
  cross_bconv_plan* ks_bconv;
  cross_bconv_plan down_bconv;  /* P -> the owned Q' limbs; NULL when nq = 0   */
} cross_hemul_shard_desc;

int cross_hemul_shard_create(const cross_hemul_shard_desc* desc, cross_hemul_shard* out);
int cross_hemul_shard_destroy(cross_hemul_shard shard);
size_t cross_hemul_shard_workspace_size(cross_hemul_shard shard, int64_t batch);
int cross_hemul_shard_modup_input(cross_hemul_shard shard, const uint32_t* in, int64_t batch, uint32_t* cc_out,
                                  void* workspace, size_t workspace_bytes, void* stream);
int cross_hemul_shard_keyswitch(cross_hemul_shard shard, const uint32_t* cc_all, int64_t batch, uint32_t* kp_out,
                                void* workspace, size_t workspace_bytes, void* stream);
int cross_hemul_shard_moddown(cross_hemul_shard shard, const uint32_t* kp_all, int64_t batch, uint32_t* out,
                              void* workspace, size_t workspace_bytes, void* stream);

/* ------------------------------------------------------------------ */
/* HE-Rotate (herot.py)                                                */
/* ------------------------------------------------------------------ */

typedef struct cross_herot_desc {
  int r, c;            /* input degree layout (only N = r*c matters)                 */
  int L, K, dnum;
  /* plan over Q then P with the default factorisation (herot.py:160-175 build every
   * Ciphertext without a finite_field_context)                                       */
  cross_ntt_plan ntt_qp;
  cross_bconv_plan* ks_bconv;     /* dnum controls: digit j -> complement in Q + P    */
  cross_bconv_plan down_bconv;    /* P -> Q                                           */
  const uint32_t* inv_psi_q;      /* (L, N)                                           */
  const uint32_t* psi_qp;         /* (L+K, N)                                         */
  const uint32_t* inv_psi_p;      /* (K, N)                                           */
  const uint32_t* p_inv_mod_q;    /* (L)                                              */
} cross_herot_desc;

int cross_herot_plan_create(const cross_herot_desc* desc, cross_herot_plan* out);
/* HERot.setup_rotate (herot.py:178-181): evk (dnum, N, L+K) host arrays and the
 * coefficient map (N) host int32 array. */
int cross_herot_set_keys(cross_herot_plan plan, const uint32_t* evk_a, const uint32_t* evk_b,
                         const int32_t* coef_map);
int cross_herot_plan_destroy(cross_herot_plan plan);
size_t cross_herot_workspace_size(cross_herot_plan plan, int64_t batch, int layout);
/* HERot.rotate (herot.py:183-302): in (batch, 2, r, c, L) -> out (batch, 2, N, L)
 * (limb-major: (batch, 2, L, N) -> (batch, 2, L, N)). */
int cross_herot(cross_herot_plan plan, const uint32_t* in, uint32_t* out, int64_t batch, int layout,
                void* workspace, size_t workspace_bytes, void* stream);

#ifdef __cplusplus
}  /* extern "C" */
#endif

#endif  /* CROSS_B200_H_ */
