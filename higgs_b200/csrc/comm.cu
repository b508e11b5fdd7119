// comm.cu -- tensor-parallel collectives over NVLink peer memory.
//
// The reference runs on one device; the tensor-parallel split of its decode
// step (column-parallel q|k|v, gate|up and LM head, row-parallel o_proj and
// down_proj) needs one sum over ranks after each row-parallel GEMV and one
// argmax over the vocabulary shards at the end.  These are tiny (B x hidden
// f32 values per call), so they are latency problems: a one-shot push over
// peer memory beats a ring.  Every rank owns one buffer, shared with the other
// ranks through CUDA IPC handles:
//
//   flags [calls][world][ctas] u32 | data [calls][world][words] u32
//
// Call j of a step writes its slice into slot (j, my rank) of every rank's
// buffer, then raises flag (j, my rank, cta) on every rank to the step number;
// each CTA waits until the flags of all ranks for its slice carry the step
// number, then reduces the slots in rank order (identical bits on all ranks).
// A call site owns its region for the whole step, so no rank can overwrite a
// region another rank is still reading: reaching call j of step s+1 requires
// every rank's flags of calls j+1.. of step s.  Spins are bounded: after about
// a second without progress the kernel records an error and finishes.
#include <cstring>

#include "common.cuh"
#include "kernels.cuh"

struct higgs_comm {
  int device = 0, rank = 0, world = 1;
  int n_calls = 0, max_ctas = 0;
  size_t words = 0;  // u32 words per slot
  size_t flag_bytes = 0;
  void* buf = nullptr;
  size_t buf_bytes = 0;
  void* peer[higgs::kMaxRanks] = {};
  unsigned* step = nullptr;  // device counter, one per rank
  int* err = nullptr;        // device error flag
};

namespace higgs {

namespace {

constexpr int kCommThreads = 512;

struct CommArgs {
  char* peer[kMaxRanks];
  int rank, world, max_ctas;
  size_t flag_bytes, words;
  const unsigned* step;
  int* err;
};

__device__ __forceinline__ void st_release_sys(unsigned* p, unsigned v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ unsigned ld_acquire_sys(const unsigned* p) {
  unsigned v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

enum { AR_SUM_RESIDUAL = 0, AR_ARGMAX = 1 };

// MODE AR_SUM_RESIDUAL: src f32 [n], h bf16 [n] in place: h = bf16(h + bf16(sum_q src_q)).
// MODE AR_ARGMAX: src u64 keys [n], out int32 [n] = ~low32(max_q key_q).
template <int MODE>
__global__ void __launch_bounds__(kCommThreads) allreduce_kernel(CommArgs c, int call, const void* src,
                                                                 int n, void* out) {
  pdl_wait();
  const unsigned s = *c.step;
  const int n_words = MODE == AR_SUM_RESIDUAL ? n : 2 * n;
  // slice of this CTA, a multiple of 4 words (16 bytes)
  const int per = ((n_words + gridDim.x - 1) / gridDim.x + 3) & ~3;
  const int w0 = blockIdx.x * per, w1 = min(n_words, w0 + per);
  const uint32_t* sw = static_cast<const uint32_t*>(src);
  for (int q = 0; q < c.world; ++q) {
    uint32_t* dst = reinterpret_cast<uint32_t*>(c.peer[q] + c.flag_bytes) +
                    ((size_t)call * c.world + c.rank) * c.words;
    for (int i = w0 + 4 * threadIdx.x; i < w1; i += 4 * kCommThreads) {
      if (i + 4 <= w1) {
        *reinterpret_cast<uint4*>(dst + i) = *reinterpret_cast<const uint4*>(sw + i);
      } else {
        for (int e = i; e < w1; ++e) dst[e] = sw[e];
      }
    }
  }
  // the barrier orders every thread's pushes before the flag writers; one system-scope
  // fence per flag writer then publishes them (measured: per-thread fences cost ~3 us a call)
  __syncthreads();
  if (threadIdx.x < c.world) {
    __threadfence_system();
    unsigned* f = reinterpret_cast<unsigned*>(c.peer[threadIdx.x]) +
                  ((size_t)call * c.world + c.rank) * c.max_ctas + blockIdx.x;
    st_release_sys(f, s);
  }
  if (threadIdx.x < c.world) {
    const unsigned* f = reinterpret_cast<const unsigned*>(c.peer[c.rank]) +
                        ((size_t)call * c.world + threadIdx.x) * c.max_ctas + blockIdx.x;
    const long long t0 = clock64();
    while (ld_acquire_sys(f) != s) {
      if (clock64() - t0 > (1ll << 31)) {  // ~1 s at 2 GHz: give up, record it
        atomicExch(c.err, 1);
        break;
      }
      __nanosleep(64);
    }
  }
  __syncthreads();
  pdl_launch();
  const uint32_t* mine = reinterpret_cast<const uint32_t*>(c.peer[c.rank] + c.flag_bytes) +
                         (size_t)call * c.world * c.words;
  if (MODE == AR_SUM_RESIDUAL) {
    // 4 words per thread: every rank's partial and the residual are loaded together (one
    // round trip), then summed in rank order -- the same bits as one element at a time
    // (the residual is read 8 bytes at a time only when it is 8-byte aligned; slots always are)
    uint16_t* h = static_cast<uint16_t*>(out);
    const bool h8 = (reinterpret_cast<uintptr_t>(h) & 7) == 0;
    for (int i = w0 + 4 * threadIdx.x; i < w1; i += 4 * kCommThreads) {
      if (h8 && i + 4 <= w1) {
        float4 v[kMaxRanks];
#pragma unroll
        for (int q = 0; q < kMaxRanks; ++q)
          if (q < c.world) v[q] = __ldcg(reinterpret_cast<const float4*>(mine + (size_t)q * c.words + i));
        const uint2 hv = *reinterpret_cast<const uint2*>(h + i);
        float y[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
        for (int q = 0; q < kMaxRanks; ++q)
          if (q < c.world) {
            y[0] += v[q].x;
            y[1] += v[q].y;
            y[2] += v[q].z;
            y[3] += v[q].w;
          }
        const uint32_t w0v = ((uint32_t)f2bf(bf2f((uint16_t)(hv.x & 0xFFFF)) + round_bf(y[0]))) |
                             ((uint32_t)f2bf(bf2f((uint16_t)(hv.x >> 16)) + round_bf(y[1])) << 16);
        const uint32_t w1v = ((uint32_t)f2bf(bf2f((uint16_t)(hv.y & 0xFFFF)) + round_bf(y[2]))) |
                             ((uint32_t)f2bf(bf2f((uint16_t)(hv.y >> 16)) + round_bf(y[3])) << 16);
        *reinterpret_cast<uint2*>(h + i) = make_uint2(w0v, w1v);
      } else {
        for (int e = i; e < min(i + 4, w1); ++e) {
          float y = 0.f;
          for (int q = 0; q < c.world; ++q) y += __uint_as_float(__ldcg(mine + (size_t)q * c.words + e));
          h[e] = f2bf(bf2f(h[e]) + round_bf(y));
        }
      }
    }
  } else {
    int32_t* o = static_cast<int32_t*>(out);
    for (int i = (w0 >> 1) + threadIdx.x; i < (w1 >> 1); i += kCommThreads) {
      unsigned long long best = 0ull;
      for (int q = 0; q < c.world; ++q) {
        const uint32_t* p = mine + (size_t)q * c.words + 2 * i;
        const unsigned long long k =
            (unsigned long long)__ldcg(p) | ((unsigned long long)__ldcg(p + 1) << 32);
        best = max(best, k);
      }
      o[i] = (int32_t)(0xFFFFFFFFu - (uint32_t)(best & 0xFFFFFFFFull));
    }
  }
}

__global__ void comm_step_kernel(unsigned* step) {
  pdl_wait();
  if (threadIdx.x == 0) *step += 1;
  pdl_launch();
}

CommArgs comm_args(const higgs_comm* c) {
  CommArgs a{};
  for (int q = 0; q < c->world; ++q) a.peer[q] = static_cast<char*>(c->peer[q]);
  a.rank = c->rank;
  a.world = c->world;
  a.max_ctas = c->max_ctas;
  a.flag_bytes = c->flag_bytes;
  a.words = c->words;
  a.step = c->step;
  a.err = c->err;
  return a;
}

int comm_ctas(const higgs_comm* c, int n_words) {
  int k = (n_words + 2047) / 2048;
  if (k < 1) k = 1;
  if (k > c->max_ctas - 2) k = c->max_ctas - 2;  // the last two flag words belong to TpFuse
  return k;
}

}  // namespace

TpFuse comm_tp_fuse(const higgs_comm* c, int call) {
  TpFuse t{};
  for (int q = 0; q < c->world; ++q) t.peer[q] = static_cast<char*>(c->peer[q]);
  t.rank = c->rank;
  t.world = c->world;
  t.call = call;
  t.max_ctas = c->max_ctas;
  t.flag_bytes = c->flag_bytes;
  t.words = c->words;
  t.step = c->step;
  t.err = c->err;
  return t;
}

cudaError_t comm_step(higgs_comm* c, cudaStream_t st) {
  return launch_pdl(comm_step_kernel, dim3(1), dim3(32), 0, st, c->step);
}

cudaError_t comm_allreduce_residual(higgs_comm* c, int call, const float* partial, int n, uint16_t* h,
                                    cudaStream_t st) {
  if (call < 0 || call >= c->n_calls || (size_t)n > c->words) return cudaErrorInvalidValue;
  return launch_pdl(allreduce_kernel<AR_SUM_RESIDUAL>, dim3(comm_ctas(c, n)), dim3(kCommThreads), 0,
                    st, comm_args(c), call, (const void*)partial, n, (void*)h);
}

cudaError_t comm_allreduce_argmax(higgs_comm* c, int call, const unsigned long long* keys, int n,
                                  int32_t* out, cudaStream_t st) {
  if (call < 0 || call >= c->n_calls || (size_t)2 * n > c->words) return cudaErrorInvalidValue;
  return launch_pdl(allreduce_kernel<AR_ARGMAX>, dim3(comm_ctas(c, 2 * n)), dim3(kCommThreads), 0, st,
                    comm_args(c), call, (const void*)keys, n, (void*)out);
}

}  // namespace higgs

using namespace higgs;

extern "C" int higgs_comm_create(higgs_ctx* ctx, int rank, int world, size_t words_per_call,
                                 int n_calls, higgs_comm** out, void* ipc_handle_out) {
  HG_CHECK_ARG(ctx && out && ipc_handle_out, "higgs_comm_create: null argument");
  HG_DEVICE(ctx);
  *out = nullptr;
  HG_CHECK_ARG(world >= 1 && world <= kMaxRanks && rank >= 0 && rank < world,
               "higgs_comm_create: bad rank / world (world <= 8)");
  HG_CHECK_ARG(words_per_call > 0 && n_calls > 0, "higgs_comm_create: empty communicator");
  higgs_comm* c = new higgs_comm;
  c->device = ctx->device;
  c->rank = rank;
  c->world = world;
  c->n_calls = n_calls;
  c->max_ctas = 32;
  c->words = (words_per_call + 3) & ~(size_t)3;
  c->flag_bytes = ((size_t)n_calls * world * c->max_ctas * 4 + 255) & ~(size_t)255;
  c->buf_bytes = c->flag_bytes + (size_t)n_calls * world * c->words * 4;
  cudaError_t e = cudaMalloc(&c->buf, c->buf_bytes);
  if (e == cudaSuccess) e = cudaMemset(c->buf, 0, c->buf_bytes);
  if (e == cudaSuccess) e = cudaMalloc(&c->step, 256);
  if (e == cudaSuccess) e = cudaMemset(c->step, 0, 256);
  if (e == cudaSuccess) c->err = reinterpret_cast<int*>(reinterpret_cast<char*>(c->step) + 128);
  cudaIpcMemHandle_t hdl;
  if (e == cudaSuccess) e = cudaIpcGetMemHandle(&hdl, c->buf);
  if (e != cudaSuccess) {
    if (c->buf) cudaFree(c->buf);
    if (c->step) cudaFree(c->step);
    delete c;
    return cuda_fail(e, "higgs_comm_create");
  }
  memcpy(ipc_handle_out, &hdl, sizeof(hdl));
  c->peer[rank] = c->buf;
  *out = c;
  return HIGGS_OK;
}

extern "C" int higgs_comm_connect(higgs_comm* c, const void* handles) {
  HG_CHECK_ARG(c && handles, "higgs_comm_connect: null argument");
  HG_DEVICE(c);
  const char* hs = static_cast<const char*>(handles);
  for (int q = 0; q < c->world; ++q) {
    if (q == c->rank) continue;
    cudaIpcMemHandle_t h;
    memcpy(&h, hs + (size_t)q * sizeof(cudaIpcMemHandle_t), sizeof(h));
    void* p = nullptr;
    HG_CUDA(cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess));
    c->peer[q] = p;
  }
  return HIGGS_OK;
}

extern "C" int higgs_comm_destroy(higgs_comm* c) {
  if (!c) return HIGGS_OK;
  DeviceGuard guard;
  guard.enter(c->device);
  for (int q = 0; q < c->world; ++q)
    if (q != c->rank && c->peer[q]) cudaIpcCloseMemHandle(c->peer[q]);
  if (c->buf) cudaFree(c->buf);
  if (c->step) cudaFree(c->step);
  delete c;
  return HIGGS_OK;
}

extern "C" size_t higgs_comm_handle_size(void) { return sizeof(cudaIpcMemHandle_t); }

extern "C" int higgs_comm_error(higgs_comm* c, int* out) {
  HG_CHECK_ARG(c && out, "higgs_comm_error: null argument");
  HG_DEVICE(c);
  int v = 0;
  HG_CUDA(cudaMemcpy(&v, c->err, sizeof(int), cudaMemcpyDeviceToHost));
  *out = v;
  if (v) HG_CUDA(cudaMemset(c->err, 0, sizeof(int)));
  return HIGGS_OK;
}

extern "C" int higgs_comm_step(higgs_comm* c, void* stream) {
  HG_CHECK_ARG(c, "higgs_comm_step: null communicator");
  HG_DEVICE(c);
  HG_CUDA(comm_step(c, (cudaStream_t)stream));
  return HIGGS_OK;
}

extern "C" int higgs_allreduce_residual(higgs_comm* c, int call, const float* partial, int n,
                                        void* h, void* stream) {
  HG_CHECK_ARG(c && partial && h && n >= 0, "higgs_allreduce_residual: bad argument");
  HG_CHECK_ARG(call >= 0 && call < c->n_calls && (size_t)n <= c->words,
               "higgs_allreduce_residual: call index or size outside the communicator");
  HG_CHECK_ARG(((uintptr_t)partial & 15) == 0, "higgs_allreduce_residual: partial must be 16-byte aligned");
  HG_DEVICE(c);
  if (n == 0) return HIGGS_OK;
  HG_CUDA(comm_allreduce_residual(c, call, partial, n, (uint16_t*)h, (cudaStream_t)stream));
  return HIGGS_OK;
}

extern "C" int higgs_allreduce_argmax(higgs_comm* c, int call, const uint64_t* keys, int n,
                                      int32_t* out, void* stream) {
  HG_CHECK_ARG(c && keys && out && n >= 0, "higgs_allreduce_argmax: bad argument");
  HG_CHECK_ARG(call >= 0 && call < c->n_calls && (size_t)2 * n <= c->words,
               "higgs_allreduce_argmax: call index or size outside the communicator");
  HG_CHECK_ARG(((uintptr_t)keys & 15) == 0, "higgs_allreduce_argmax: keys must be 16-byte aligned");
  HG_DEVICE(c);
  if (n == 0) return HIGGS_OK;
  HG_CUDA(comm_allreduce_argmax(c, call, (const unsigned long long*)keys, n, out,
                                (cudaStream_t)stream));
  return HIGGS_OK;
}
