// Shared plumbing for the joyomni_b200 C-ABI library: status codes, the
// thread-local last-error string, dtype tags and 16-byte vector helpers.
//
// Error convention (mirrors the reference's TORCH_CHECK / JO_CHECK_* behaviour,
// deploy/joyomni_ops/include/joyomni_ops.h:8-15): every entry point validates
// its arguments, returns a negative status on failure and leaves a message in
// jo_last_error().  The Python shim turns JO_ERR_ARCH into NotImplementedError
// (as TORCH_CHECK_NOT_IMPLEMENTED does, fp8_gemm.cu:1531) and everything else
// into RuntimeError.
#pragma once

#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_fp8.h>
#include <stdint.h>
#include <stdarg.h>
#include <stdio.h>

#include "../../include/joyomni_b200.h"

namespace jo {

// ---------------------------------------------------------------- errors ----
void set_error(const char* fmt, ...);

#define JO_REQUIRE(cond, code, ...)      \
  do {                                   \
    if (!(cond)) {                       \
      ::jo::set_error(__VA_ARGS__);      \
      return (code);                     \
    }                                    \
  } while (0)

// Checks that the current device is sm_100 (B200 class).  Cached per device.
int require_sm100();

// Checks the last launch; converts a CUDA error into JO_ERR_CUDA.
int check_launch(const char* what);

// Number of SMs of the current device (cached).
int sm_count();

// Launch-configuration caches (shared-memory opt-ins, occupancy) are kept per
// device, since a process may launch on several GPUs.
constexpr int kMaxDevices = 64;
// Index of the current device, clamped into [0, kMaxDevices).
inline int device_slot() {
  int d = 0;
  if (cudaGetDevice(&d) != cudaSuccess) {
    cudaGetLastError();
    d = 0;
  }
  return d < 0 ? 0 : d % kMaxDevices;
}

inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }
inline bool aligned8(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 7u) == 0; }

// ------------------------------------------------------------- dtypes ------
template <int DT> struct Elem;
template <> struct Elem<JO_DTYPE_F32> { using T = float; };
template <> struct Elem<JO_DTYPE_F16> { using T = __half; };
template <> struct Elem<JO_DTYPE_BF16> { using T = __nv_bfloat16; };

__device__ __forceinline__ float to_f32(float v) { return v; }
__device__ __forceinline__ float to_f32(__half v) { return __half2float(v); }
__device__ __forceinline__ float to_f32(__nv_bfloat16 v) { return __bfloat162float(v); }

template <typename T> __device__ __forceinline__ T from_f32(float v);
template <> __device__ __forceinline__ float from_f32<float>(float v) { return v; }
template <> __device__ __forceinline__ __half from_f32<__half>(float v) { return __float2half_rn(v); }
template <> __device__ __forceinline__ __nv_bfloat16 from_f32<__nv_bfloat16>(float v) {
  return __float2bfloat16_rn(v);
}

// A 16-byte vector of elements of T (8 x bf16/fp16 or 4 x fp32).
template <typename T>
struct Vec16 {
  static constexpr int N = 16 / sizeof(T);
  uint4 raw;
  __device__ __forceinline__ float get(int i) const {
    const T* p = reinterpret_cast<const T*>(&raw);
    return to_f32(p[i]);
  }
  __device__ __forceinline__ void set(int i, float v) {
    T* p = reinterpret_cast<T*>(&raw);
    p[i] = from_f32<T>(v);
  }
};

// Streaming 16-byte global load that does not allocate in L1 (single-use data).
__device__ __forceinline__ uint4 ld_stream(const void* p) {
  uint4 r;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
               : "l"(p));
  return r;
}
// Plain 16-byte read-only load, cached in L1 (small reused tables).
__device__ __forceinline__ uint4 ld_cached(const void* p) {
  return __ldg(reinterpret_cast<const uint4*>(p));
}
__device__ __forceinline__ void st_stream(void* p, uint4 v) {
  asm volatile("st.global.cs.v4.u32 [%0], {%1,%2,%3,%4};" ::"l"(p), "r"(v.x), "r"(v.y),
               "r"(v.z), "r"(v.w)
               : "memory");
}

__device__ __forceinline__ float warp_sum(float v, int width = 32) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1)
    if (o < width) v += __shfl_xor_sync(0xffffffffu, v, o, 32);
  return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o, 32));
  return v;
}

constexpr float kFp8Max = 448.0f;

// ---- packed 16-bit pairs ---------------------------------------------------
// One 32-bit word holds two 16-bit elements; element 0 in the low half.
template <typename T> __device__ __forceinline__ float2 unpack2(uint32_t w);
template <> __device__ __forceinline__ float2 unpack2<__nv_bfloat16>(uint32_t w) {
  return make_float2(__uint_as_float(w << 16), __uint_as_float(w & 0xffff0000u));
}
template <> __device__ __forceinline__ float2 unpack2<__half>(uint32_t w) {
  __half2 h = *reinterpret_cast<__half2*>(&w);
  return __half22float2(h);
}
template <typename T> __device__ __forceinline__ uint32_t pack2(float lo, float hi);
template <> __device__ __forceinline__ uint32_t pack2<__nv_bfloat16>(float lo, float hi) {
  uint32_t r;
  asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
  return r;
}
template <> __device__ __forceinline__ uint32_t pack2<__half>(float lo, float hi) {
  uint32_t r;
  asm("cvt.rn.f16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
  return r;
}
// Bit pattern of +inf for the 16-bit type; |x| bit patterns above it are NaN.
template <typename T> struct Bits16;
template <> struct Bits16<__nv_bfloat16> { static constexpr uint32_t kInf = 0x7f80u; };
template <> struct Bits16<__half> { static constexpr uint32_t kInf = 0x7c00u; };
template <typename T> __device__ __forceinline__ float from_bits16(uint32_t b);
template <> __device__ __forceinline__ float from_bits16<__nv_bfloat16>(uint32_t b) {
  return __uint_as_float(b << 16);
}
template <> __device__ __forceinline__ float from_bits16<__half>(uint32_t b) {
  return __half2float(__ushort_as_half((unsigned short)b));
}
// Running max of |elements| over packed pairs, on the integer bit patterns
// (for non-NaN values |x| orders like its bits; NaN patterns sort above inf).
__device__ __forceinline__ uint32_t absmax2(uint32_t acc, uint32_t w) {
  uint32_t r;
  asm("max.u16x2 %0, %1, %2;" : "=r"(r) : "r"(acc), "r"(w & 0x7fff7fffu));
  return r;
}
__device__ __forceinline__ uint32_t absmax2_fold(uint32_t acc) { return max(acc & 0xffffu, acc >> 16); }

// Running max of |elements| over packed 16-bit pairs in the floating-point
// unit: one instruction per pair.  The result's sign bits are meaningless
// (xorsign) and are masked by the fold; a NaN operand yields the canonical NaN
// (0x7fff), whose masked pattern sorts above +inf, so the caller can flag it.
template <typename T> __device__ __forceinline__ uint32_t absmax_h2(uint32_t acc, uint32_t w);
template <> __device__ __forceinline__ uint32_t absmax_h2<__nv_bfloat16>(uint32_t acc, uint32_t w) {
  uint32_t r;
  asm("max.NaN.xorsign.abs.bf16x2 %0, %1, %2;" : "=r"(r) : "r"(acc), "r"(w));
  return r;
}
template <> __device__ __forceinline__ uint32_t absmax_h2<__half>(uint32_t acc, uint32_t w) {
  uint32_t r;
  asm("max.NaN.xorsign.abs.f16x2 %0, %1, %2;" : "=r"(r) : "r"(acc), "r"(w));
  return r;
}
// Same without NaN propagation: a NaN operand yields the other operand, so the
// result is the max of |x| over the non-NaN elements (as fmaxf reductions do).
template <typename T> __device__ __forceinline__ uint32_t absmax_h2_nonan(uint32_t acc, uint32_t w);
template <> __device__ __forceinline__ uint32_t absmax_h2_nonan<__nv_bfloat16>(uint32_t acc, uint32_t w) {
  uint32_t r;
  asm("max.xorsign.abs.bf16x2 %0, %1, %2;" : "=r"(r) : "r"(acc), "r"(w));
  return r;
}
template <> __device__ __forceinline__ uint32_t absmax_h2_nonan<__half>(uint32_t acc, uint32_t w) {
  uint32_t r;
  asm("max.xorsign.abs.f16x2 %0, %1, %2;" : "=r"(r) : "r"(acc), "r"(w));
  return r;
}
__device__ __forceinline__ uint32_t absmax_h2_fold(uint32_t acc) {
  return max(acc & 0x7fffu, (acc >> 16) & 0x7fffu);
}

// ---- paired fp32 arithmetic (sm_100: one instruction, two IEEE RN lanes) ----
// Each lane is exactly the scalar fma.rn / mul.rn / add.rn of that lane.  The
// compiler builtins let the register allocator place the pairs itself.
__device__ __forceinline__ float2 fma2(float2 a, float2 b, float2 c) { return __ffma2_rn(a, b, c); }
__device__ __forceinline__ float2 mul2(float2 a, float2 b) { return __fmul2_rn(a, b); }
__device__ __forceinline__ float2 add2(float2 a, float2 b) { return __fadd2_rn(a, b); }

// a / 448 correctly rounded, for a = |x| of a 16-bit (bf16 or fp16) value:
// one multiply by RN(1/448) and one FMA correction step -- Markstein's
// residual correction (P. Markstein, "Computation of elementary functions on
// the IBM RISC System/6000 processor", IBM J. Res. Dev. 34(1), 1990): with
// q = RN(a*c), the residual r = a - q*448 is exact in one FMA, and
// RN(q + r*c) is the correctly rounded quotient when c = RN(1/448) and the
// dividend range is limited as here.  Checked exhaustively
// against the exact quotient for every finite positive bf16 and fp16 value
// (tests/test_oracle.py emulates the three roundings with exact rationals).
__device__ __forceinline__ float div448_h(float a) {
  const float c = 1.f / 448.f;  // folded to RN(1/448) at compile time
  const float q = __fmul_rn(a, c);
  const float r = __fmaf_rn(-q, 448.f, a);
  return __fmaf_rn(r, c, q);
}

// Four floats -> four e4m3 codes in one 32-bit word (element 0 in the low
// byte), round-to-nearest-even, satfinite; the two 16-bit conversion results
// are joined inside the asm block.
__device__ __forceinline__ uint32_t pack_e4m3x4(float a, float b, float c, float d) {
  uint32_t r;
  asm("{\n .reg .b16 lo, hi;\n cvt.rn.satfinite.e4m3x2.f32 lo, %2, %1;\n cvt.rn.satfinite.e4m3x2.f32 hi, %4, %3;\n"
      " mov.b32 %0, {lo, hi};\n}"
      : "=r"(r)
      : "f"(a), "f"(b), "f"(c), "f"(d));
  return r;
}

// Two floats -> two packed e4m3 codes, round-to-nearest-even, satfinite.
__device__ __forceinline__ uint16_t pack_e4m3x2(float lo, float hi) {
  __nv_fp8x2_storage_t s = __nv_cvt_float2_to_fp8x2(make_float2(lo, hi), __NV_SATFINITE, __NV_E4M3);
  return static_cast<uint16_t>(s);
}

}  // namespace jo
