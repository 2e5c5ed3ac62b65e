// Error state, device-memory helpers and the modulus-set entry points.
#include <atomic>
#include <cstdarg>
#include <cstdio>
#include <cstring>

#include "internal.hpp"

namespace cross {

static thread_local char g_err[512] = "";
static std::atomic<uint64_t> g_launches{0};

void count_launch(unsigned n) { g_launches.fetch_add(n, std::memory_order_relaxed); }

void set_error(const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_err, sizeof(g_err), fmt, ap);
  va_end(ap);
}

static int device_attr(cudaDeviceAttr attr, int fallback) {
  int d = 0, v = 0;
  if (cudaGetDevice(&d) != cudaSuccess || cudaDeviceGetAttribute(&v, attr, d) != cudaSuccess || v <= 0) {
    (void)cudaGetLastError();
    return fallback;
  }
  return v;
}
static PerDevice g_sms, g_smem;
int device_sm_count() { return g_sms.get([] { return device_attr(cudaDevAttrMultiProcessorCount, 148); }); }
int device_smem_per_sm() {
  return g_smem.get([] { return device_attr(cudaDevAttrMaxSharedMemoryPerMultiprocessor, 233472); });
}

int fail_cuda(cudaError_t e, const char* where) {
  set_error("CUDA error %d (%s) at %s", (int)e, cudaGetErrorString(e), where);
  return CROSS_ERR_CUDA;
}

template <class T>
int upload(T** dst, const T* src, size_t count) {
  *dst = nullptr;
  if (count == 0) return CROSS_OK;
  CROSS_CHECK_CUDA(cudaMalloc((void**)dst, count * sizeof(T)));
  CROSS_CHECK_CUDA(cudaMemcpy(*dst, src, count * sizeof(T), cudaMemcpyHostToDevice));
  return CROSS_OK;
}
template int upload<uint32_t>(uint32_t**, const uint32_t*, size_t);
template int upload<uint16_t>(uint16_t**, const uint16_t*, size_t);
template int upload<uint8_t>(uint8_t**, const uint8_t*, size_t);
template int upload<int16_t>(int16_t**, const int16_t*, size_t);
template int upload<int32_t>(int32_t**, const int32_t*, size_t);
template int upload<ModC>(ModC**, const ModC*, size_t);
template int upload<VarC>(VarC**, const VarC*, size_t);

// Inverse of a modulo an odd m (extended Euclid on signed 64-bit values; the
// callers keep a and m below 2^32).
static uint64_t inv_mod(uint64_t a, uint64_t m) {
  int64_t t = 0, nt = 1, r = (int64_t)m, nr = (int64_t)(a % m);
  while (nr) {
    const int64_t qt = r / nr;
    const int64_t t2 = t - qt * nt, r2 = r - qt * nr;
    t = nt; nt = t2; r = nr; nr = r2;
  }
  return (uint64_t)(t < 0 ? t + (int64_t)m : t);
}

std::vector<VarC> make_varc(const std::vector<ModC>& mods) {
  std::vector<VarC> v(mods.size());
  for (size_t i = 0; i < mods.size(); ++i) {
    const uint64_t q = mods[i].q;
    VarC& c = v[i];
    c.q = (uint32_t)q;
    // q^-1 mod 2^32 by Newton's iteration (each step doubles the correct low bits)
    uint32_t x = (uint32_t)q;
    for (int k = 0; k < 5; ++k) x *= 2u - (uint32_t)q * x;
    c.qinv = x;
    c.winv = (uint32_t)inv_mod((1ull << 32) % q, q);
    c.pad = 0;
    uint64_t p = (1ull << 32) % q;
    for (int j = 0; j < 4; ++j) {
      c.r[j] = (uint32_t)p;
      p = (p << 8) % q;
    }
  }
  return v;
}

void dfree(void* p) {
  if (p) cudaFree(p);
}

}  // namespace cross

extern "C" {

int cross_abi_version(void) { return CROSS_B200_ABI_VERSION; }

const char* cross_last_error(void) { return cross::g_err; }

uint64_t cross_launch_count(void) { return cross::g_launches.load(std::memory_order_relaxed); }

int cross_moduli_create(int num_moduli, const uint32_t* moduli, const uint64_t* barrett_m,
                        const uint32_t* barrett_w, const uint32_t* barrett_s_w, cross_moduli* out) {
  CROSS_REQUIRE(out && moduli && barrett_m && barrett_w && barrett_s_w && num_moduli > 0,
                "cross_moduli_create: null argument or num_moduli <= 0");
  *out = nullptr;
  auto* s = new cross_moduli_s();
  s->n = num_moduli;
  for (int i = 0; i < num_moduli; ++i) {
    if (moduli[i] < 3 || (moduli[i] & 1u) == 0 || moduli[i] >= (1u << 31) || barrett_w[i] > 32 ||
        barrett_s_w[i] > 63) {
      cross::set_error("cross_moduli_create: modulus %u (index %d) must be odd, in [3, 2^31)",
                       moduli[i], i);
      delete s;
      return CROSS_ERR_INVALID_ARG;
    }
    s->host.push_back(cross::ModC{moduli[i], barrett_m[i], barrett_w[i], barrett_s_w[i]});
  }
  std::vector<uint4> packed;
  for (const cross::ModC& mc : s->host)
    packed.push_back(make_uint4((uint32_t)mc.q, (uint32_t)mc.m, mc.s_w,
                                (cross::barrett_w32_ok(mc) ? 1u : 0u) | (cross::reduce_fast_ok(mc) ? 2u : 0u)));
  int rc = cross::upload_vec(&s->dev, s->host);
  if (!rc) rc = cross::upload_vec(&s->dev_v, cross::make_varc(s->host));
  if (!rc) rc = cross::upload_vec(&s->dev_f, packed);
  if (rc) {
    cross::dfree(s->dev);
    cross::dfree(s->dev_v);
    cross::dfree(s->dev_f);
    delete s;
    return rc;
  }
  *out = s;
  return CROSS_OK;
}

int cross_moduli_destroy(cross_moduli m) {
  if (!m) return CROSS_OK;
  cross::dfree(m->dev);
  cross::dfree(m->dev_v);
  cross::dfree(m->dev_f);
  delete m;
  return CROSS_OK;
}

}  // extern "C"
