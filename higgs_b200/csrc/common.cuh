// common.cuh -- shared device/host helpers for the higgs sm_100a kernels.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <string>

#include "../../include/higgs_cuda.h"

namespace higgs {

// ---------------------------------------------------------------------------
// host-side error plumbing (thread-local message behind higgs_last_error())
// ---------------------------------------------------------------------------
void set_error(const std::string& msg);
int fail(int code, const std::string& msg);
int cuda_fail(cudaError_t e, const char* what);

#define HG_CHECK_ARG(cond, msg)                                  \
  do {                                                           \
    if (!(cond)) return ::higgs::fail(HIGGS_ERR_INVALID_ARG, msg); \
  } while (0)

#define HG_CUDA(call)                                          \
  do {                                                         \
    cudaError_t e_ = (call);                                   \
    if (e_ != cudaSuccess) return ::higgs::cuda_fail(e_, #call); \
  } while (0)

// Launch with programmatic dependent launch enabled: the kernel may begin
// (and prefetch weights that do not depend on the previous kernel) while the
// previous kernel on the stream drains; it calls pdl_wait() before touching
// anything the previous kernel wrote.  Works inside stream capture.
template <typename... KArgs, typename... Args>
cudaError_t launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem,
                       cudaStream_t stream, Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kernel, static_cast<KArgs>(args)...);
}

// ---------------------------------------------------------------------------
// per-device state
// ---------------------------------------------------------------------------
// A process may hold contexts on several GPUs.  Every entry point that takes a
// context (or a model / communicator built on one) makes that context's
// device current for the duration of the call (DeviceGuard), so helpers below
// it can key their state on the current device.  Device-side state (the
// tensor-core matmul's timeout flag) is allocated by higgs_init, once per
// device; nothing allocates lazily inside a compute call.
constexpr int kMaxDevices = 64;

struct DeviceState {
  int sms = 0;            // multiprocessor count
  int* tc_err = nullptr;  // tensor-core matmul timeout flag (device int)
};

// State of device `dev` (0 <= dev < kMaxDevices); filled by higgs_init.
DeviceState& device_state(int dev);

// launch_pdl with a thread-block cluster of cluster_x CTAs along x
template <typename... KArgs, typename... Args>
cudaError_t launch_pdl_cluster(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem,
                               cudaStream_t stream, int cluster_x, Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  attr[1].id = cudaLaunchAttributeClusterDimension;
  attr[1].val.clusterDim.x = cluster_x;
  attr[1].val.clusterDim.y = 1;
  attr[1].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 2;
  return cudaLaunchKernelEx(&cfg, kernel, static_cast<KArgs>(args)...);
}

inline int current_device() {
  int d = 0;
  if (cudaGetDevice(&d) != cudaSuccess || d < 0 || d >= kMaxDevices) d = 0;
  return d;
}

inline int sm_count() {
  const int n = device_state(current_device()).sms;
  return n > 0 ? n : 148;
}

// A one-time host action (a kernel attribute) done once per device: a kernel's
// dynamic shared-memory limit is a per-device setting.  Two threads may both
// run the action the first time; it is idempotent.
struct PerDeviceOnce {
  unsigned long long done = 0;
  template <typename Fn>
  cudaError_t run(Fn fn) {
    const unsigned long long bit = 1ull << current_device();
    if (__atomic_load_n(&done, __ATOMIC_ACQUIRE) & bit) return cudaSuccess;
    const cudaError_t e = fn();
    if (e == cudaSuccess) __atomic_fetch_or(&done, bit, __ATOMIC_ACQ_REL);
    return e;
  }
};

// Makes `dev` current for one entry-point call and restores the caller's
// device on return.
class DeviceGuard {
 public:
  DeviceGuard() = default;
  DeviceGuard(const DeviceGuard&) = delete;
  DeviceGuard& operator=(const DeviceGuard&) = delete;
  int enter(int dev) {
    int cur = -1;
    cudaError_t e = cudaGetDevice(&cur);
    if (e != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
    if (cur == dev) return 0;
    e = cudaSetDevice(dev);
    if (e != cudaSuccess) return cuda_fail(e, "cudaSetDevice(context device)");
    prev_ = cur;
    return 0;
  }
  ~DeviceGuard() {
    if (prev_ >= 0) cudaSetDevice(prev_);
  }

 private:
  int prev_ = -1;
};

}  // namespace higgs

struct higgs_ctx {
  int device;
  int sms;
};

namespace higgs {

// First statement of an entry point after its null checks: run on ctx's device.
#define HG_DEVICE(ctx_)                                               \
  ::higgs::DeviceGuard hg_device_guard_;                              \
  do {                                                                \
    const int hg_e_ = hg_device_guard_.enter((ctx_)->device);         \
    if (hg_e_ != 0) return hg_e_;                                     \
  } while (0)

// ---------------------------------------------------------------------------
// device helpers
// ---------------------------------------------------------------------------
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_launch() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

__device__ __forceinline__ float bf2f(uint16_t h) { return __uint_as_float((uint32_t)h << 16); }
__device__ __forceinline__ uint16_t f2bf(float f) {
  return __bfloat16_as_ushort(__float2bfloat16_rn(f));
}
__device__ __forceinline__ float round_bf(float f) { return bf2f(f2bf(f)); }
__device__ __forceinline__ float bf_lo(uint32_t v) { return __uint_as_float(v << 16); }
__device__ __forceinline__ float bf_hi(uint32_t v) { return __uint_as_float(v & 0xffff0000u); }
__device__ __forceinline__ uint32_t pack_bf2(float lo, float hi) {
  return (uint32_t)f2bf(lo) | ((uint32_t)f2bf(hi) << 16);
}

// (x0, x1) as bf16 pairs hi = bf16(x), lo = bf16(x - hi): hi + lo carries ~16
// mantissa bits, so two bf16 MMAs reproduce an f32 operand closely.
__device__ __forceinline__ void split_bf2(float x0, float x1, uint32_t& hi, uint32_t& lo) {
  hi = pack_bf2(x0, x1);
  lo = pack_bf2(x0 - bf_lo(hi), x1 - bf_hi(hi));
}

// (a & b) | c in one LOP3
__device__ __forceinline__ uint32_t lop3_and_or(uint32_t a, uint32_t b, uint32_t c) {
  uint32_t d;
  asm("lop3.b32 %0, %1, %2, %3, 0xEA;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
  return d;
}

// Two 4-bit codes (nibbles i and i+4 of w after a right shift by 4*i) as the
// bf16 pair (128 + q_i, 128 + q_{i+4}); exact, since 128..143 are bf16 values.
template <int SHIFT>
__device__ __forceinline__ uint32_t nib_pair_bf16(uint32_t w) {
  return lop3_and_or(w >> SHIFT, 0x000F000Fu, 0x43004300u);
}

__device__ __forceinline__ uint32_t prmt(uint32_t a, uint32_t b, uint32_t sel) {
  uint32_t d;
  asm("prmt.b32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(sel));
  return d;
}

// D = A(16x16 bf16, row) * B(16x8 bf16, col) + C (f32)
__device__ __forceinline__ void mma_bf16_16816(float (&d)[4], uint32_t a0, uint32_t a1,
                                               uint32_t a2, uint32_t a3, uint32_t b0,
                                               uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
      "{%8,%9}, {%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

__device__ __forceinline__ uint2 ldg_stream_u2(const void* p) {
  uint2 v;
  asm volatile("ld.global.nc.L1::no_allocate.v2.u32 {%0,%1}, [%2];"
               : "=r"(v.x), "=r"(v.y)
               : "l"(p));
  return v;
}

__device__ __forceinline__ uint4 ldg_stream_u4(const void* p) {
  uint4 v;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p));
  return v;
}

__device__ __forceinline__ uint4 ldg_u4(const void* p) {
  return *reinterpret_cast<const uint4*>(p);
}

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void cp_async16(void* smem, const void* gmem) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(smem)), "l"(gmem));
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N));
}

__device__ __forceinline__ void ldmatrix_x4(uint32_t (&r)[4], const void* p) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(smem_u32(p)));
}
__device__ __forceinline__ void ldmatrix_x4_trans(uint32_t (&r)[4], const void* p) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(smem_u32(p)));
}

// exp(x) from correctly rounded f32 operations only (Cody-Waite reduction by
// ln 2, degree-7 Taylor polynomial, exponent scaling), so host code performing
// the same operations gets the same bits.
__device__ __forceinline__ float det_exp(float x) {
  if (!(x >= -87.0f)) return 0.0f;
  if (x > 88.0f) x = 88.0f;
  const float kf = rintf(__fmul_rn(x, 1.44269504088896341f));
  float r = __fmaf_rn(-kf, 0.693145751953125f, x);
  r = __fmaf_rn(-kf, 1.42860682030941723e-6f, r);
  float p = 1.98412698412698413e-4f;
  p = __fmaf_rn(p, r, 1.38888888888888889e-3f);
  p = __fmaf_rn(p, r, 8.33333333333333333e-3f);
  p = __fmaf_rn(p, r, 4.16666666666666667e-2f);
  p = __fmaf_rn(p, r, 1.66666666666666667e-1f);
  p = __fmaf_rn(p, r, 0.5f);
  p = __fmaf_rn(p, r, 1.0f);
  p = __fmaf_rn(p, r, 1.0f);
  const int k = (int)kf;
  return __fmul_rn(p, __uint_as_float((uint32_t)(k + 127) << 23));
}

// Orderable u64 key for argmax-style reductions: (ordered value bits << 32) |
// (~index), so the u64 maximum is the largest value and, among equal values,
// the lowest index.  NaN maps to the smallest key; -0 is folded onto +0.
__device__ __forceinline__ unsigned long long argmax_key(float v, int j) {
  uint32_t u = __float_as_uint(v);
  if (v == 0.0f) u = 0u;
  const uint32_t o = (v != v) ? 0u : ((u & 0x80000000u) ? ~u : (u | 0x80000000u));
  return ((unsigned long long)o << 32) | (unsigned long long)(0xFFFFFFFFu - (uint32_t)j);
}

// ---------------------------------------------------------------------------
// L2 prefetch of read-only ranges (weights) by the TMA unit
// ---------------------------------------------------------------------------
// Ranges a later kernel of the step will stream: every CTA of the current
// kernel asks for its share of their union with cp.async.bulk.prefetch.L2
// before it waits on its predecessor, so HBM keeps streaming weights while the
// step's dependency chain runs.  A prefetch is only a hint: it changes no data.
// Ranges start on 16-byte boundaries and are whole multiples of 16 bytes.
struct L2Prefetch {
  static constexpr int kMax = 12;
  const void* ptr[kMax];
  unsigned long long bytes[kMax];
  int n;
};

__device__ __forceinline__ void l2_prefetch_bulk(const void* p, uint32_t bytes) {
  asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(p), "r"(bytes) : "memory");
}

// one lane walks [p, p + bytes) in 32 KB requests
__device__ __forceinline__ void l2_prefetch_range(const void* p, unsigned long long bytes) {
  if ((reinterpret_cast<uintptr_t>(p) & 15) != 0) return;  // the bulk unit needs 16-byte alignment
  bytes &= ~15ull;
  const char* c = static_cast<const char*>(p);
  for (unsigned long long o = 0; o < bytes; o += 32768)
    l2_prefetch_bulk(c + o, (uint32_t)(bytes - o < 32768 ? bytes - o : 32768));
}

// Share `cta` of `ncta` of the union of the ranges, issued by the lanes of warp 0.
__device__ __forceinline__ void issue_l2_prefetch(const L2Prefetch& pf, int cta, int ncta) {
  if (pf.n <= 0 || threadIdx.x >= 32) return;
  unsigned long long total = 0;
  for (int i = 0; i < pf.n; ++i) total += pf.bytes[i];
  const unsigned long long per = ((total + ncta - 1) / ncta + 15) & ~15ull;
  const unsigned long long lo = (unsigned long long)cta * per;
  const unsigned long long hi = lo + per < total ? lo + per : total;
  unsigned long long base = 0;
  for (int i = 0; i < pf.n; ++i) {
    const unsigned long long b0 = base, b1 = base + pf.bytes[i];
    base = b1;
    const unsigned long long s = lo > b0 ? lo : b0, e = hi < b1 ? hi : b1;
    if (s >= e || ((reinterpret_cast<uintptr_t>(pf.ptr[i]) | pf.bytes[i]) & 15) != 0) continue;
    const char* c = static_cast<const char*>(pf.ptr[i]) + (s - b0);
    const unsigned long long len = e - s;
    for (unsigned long long o = (unsigned long long)threadIdx.x * 32768; o < len; o += 32 * 32768ull)
      l2_prefetch_bulk(c + o, (uint32_t)(len - o < 32768 ? len - o : 32768));
  }
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

}  // namespace higgs
