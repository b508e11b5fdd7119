// timeline.cuh -- optional per-CTA timestamps of the decode-step kernels.
//
// Compiled in only when HIGGS_TIMELINE is defined (the diagnostic library built by
// `python -m higgs_b200.build --timeline`); otherwise every macro is empty and the
// kernels are unchanged.  Thread 0 of each CTA reads %globaltimer (ns, one clock
// for the whole GPU) at marks 0 (entry), 1 (past griddepcontrol.wait) and up to
// three kernel-specific phase marks (4, 5, 6), and at exit appends one record.
// Each translation unit that includes this header keeps its own record buffer
// and exports its own fetch function, so no relocatable device code is needed.
#pragma once

#ifdef HIGGS_TIMELINE
namespace higgs {
namespace tl {

struct Rec {
  unsigned long long tag_grid;  // tag << 32 | CTAs in the grid
  unsigned long long blk_sm;    // linear CTA index << 32 | SM id
  unsigned long long t0, t1, t2, m4, m5, m6;
};
constexpr int kMax = 1 << 19;
static __device__ Rec g_rec[kMax];
static __device__ unsigned g_n;

__device__ __forceinline__ unsigned long long now() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}
__device__ __forceinline__ unsigned long long* marks() {
  __shared__ unsigned long long s[8];
  return s;
}
__device__ __forceinline__ void mark(int i) {
  if (threadIdx.x == 0) marks()[i] = now();
}
__device__ __forceinline__ void put(unsigned tag) {
  if (threadIdx.x != 0) return;
  const unsigned long long t2 = now();
  unsigned smid;
  asm("mov.u32 %0, %%smid;" : "=r"(smid));
  const unsigned i = atomicAdd(&g_n, 1u);
  if (i >= (unsigned)kMax) return;
  const unsigned long long* s = marks();
  Rec r;
  r.tag_grid = ((unsigned long long)tag << 32) | (gridDim.x * gridDim.y * gridDim.z);
  r.blk_sm = ((unsigned long long)(blockIdx.x + gridDim.x * (blockIdx.y + gridDim.y * blockIdx.z)) << 32) | smid;
  r.t0 = s[0];
  r.t1 = s[1];
  r.t2 = t2;
  r.m4 = s[4];
  r.m5 = s[5];
  r.m6 = s[6];
  g_rec[i] = r;
}

}  // namespace tl
}  // namespace higgs

#define HG_TL_MARK(i) ::higgs::tl::mark(i)
#define HG_TL_END(tag) ::higgs::tl::put(tag)
// copies up to max records (64 bytes each) to host memory out (null: count only), returns
// the count, and clears the buffer when reset is nonzero
#define HG_TL_FETCH_FN(name)                                                              \
  extern "C" int name(void* out, int max, int reset) {                                    \
    unsigned n = 0;                                                                       \
    if (cudaMemcpyFromSymbol(&n, ::higgs::tl::g_n, sizeof(n)) != cudaSuccess) return -1;  \
    if (n > (unsigned)::higgs::tl::kMax) n = ::higgs::tl::kMax;                           \
    if ((int)n > max) n = max;                                                            \
    if (out && n &&                                                                       \
        cudaMemcpyFromSymbol(out, ::higgs::tl::g_rec, n * sizeof(::higgs::tl::Rec)) != cudaSuccess) \
      return -1;                                                                          \
    if (reset) {                                                                          \
      const unsigned z = 0;                                                               \
      if (cudaMemcpyToSymbol(::higgs::tl::g_n, &z, sizeof(z)) != cudaSuccess) return -1;  \
    }                                                                                     \
    return (int)n;                                                                        \
  }
#else
#define HG_TL_MARK(i) \
  do {            \
  } while (0)
#define HG_TL_END(tag) \
  do {             \
  } while (0)
#define HG_TL_FETCH_FN(name)
#endif
