// kernels.cuh -- internal (C++) launch interfaces shared by the C-ABI entry
// points and the native decode-step runner.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

namespace higgs {

enum { EPI_STORE = 0, EPI_SWIGLU = 1 };

struct QLinArgs {
  const uint16_t* x;
  int M, K, N;
  const uint32_t* w;
  const uint16_t* s;
  const uint16_t* b;
  // optional row segments: rows [seg_end[i-1], seg_end[i]) come from weight i
  // (segment 0 is w/s/b); lets q|k|v run as one launch over separate tensors
  int nseg;
  int seg_end[3];
  const uint32_t* wseg[3];
  const uint16_t* sseg[3];
  const uint16_t* bseg[3];
  const uint32_t* w2;  // up projection (SwiGLU)
  const uint16_t* s2;
  const uint16_t* b2;
  uint16_t* y;
  float* y_f32;
  const uint16_t* residual;
  // optional fused RMSNorm of x (ring GEMV only): x is the residual stream h
  const uint16_t* norm_w;
  float eps;
};

// W4 GEMV with per-warp cp.async rings (any M, 32 rows per pass; norm_w needs
// qgemv_ring_can_fuse_norm(M, K)).
cudaError_t launch_qgemv_ring(const QLinArgs& a, int epi, cudaStream_t st);
bool qgemv_ring_can_fuse_norm(int M, int K);

// M may exceed 32 (processed in 32-row passes); K % 256 == 0, N % 16 == 0.
cudaError_t launch_qlinear(const QLinArgs& a, int epi, cudaStream_t st);

// Stream-K GEMV (M <= 8), optional fused RMSNorm of x with norm_w.
struct SkArgs {
  const uint16_t* x;
  const uint16_t* norm_w;
  float eps;
  int M, K, N;
  int n_tiles;  // 16-row weight tiles (SwiGLU: gate/up interleaved, 2 per output tile)
  int swiglu;
  int nseg;
  int seg_end[3];
  const uint32_t* wseg[3];
  const uint16_t* sseg[3];
  const uint16_t* bseg[3];
  uint16_t* y;
  float* y_f32;
  const uint16_t* residual;
  // filled by the launcher from the workspace
  int max_slots;
  int* counters;
  float* partials;
};
size_t qgemv_sk_workspace(int M, int K, int n_tiles);
cudaError_t launch_qgemv_sk(SkArgs a, void* workspace, cudaStream_t st);

}  // namespace higgs
