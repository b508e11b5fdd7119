// capi.cu -- context lifetime and the thread-local error channel of the C ABI.
#include <mutex>
#include <string>

#include "common.cuh"

namespace higgs {

DeviceState& device_state(int dev) {
  static DeviceState states[kMaxDevices];
  return states[(dev >= 0 && dev < kMaxDevices) ? dev : 0];
}

// Per-device set-up done by the first higgs_init on each device, with that
// device current: the multiprocessor count and the tensor-core matmul's
// timeout flag (the only device memory the library holds per device).
static int device_setup(int dev, int sms) {
  static std::mutex mu;
  std::lock_guard<std::mutex> lock(mu);
  DeviceState& st = device_state(dev);
  st.sms = sms;
  if (!st.tc_err) {
    int* p = nullptr;
    HG_CUDA(cudaMalloc(&p, sizeof(int)));
    const cudaError_t e = cudaMemset(p, 0, sizeof(int));
    if (e != cudaSuccess) {
      cudaFree(p);
      return cuda_fail(e, "cudaMemset(tensor-core error flag)");
    }
    st.tc_err = p;
  }
  return HIGGS_OK;
}

static thread_local std::string g_last_error;

void set_error(const std::string& msg) { g_last_error = msg; }

int fail(int code, const std::string& msg) {
  g_last_error = msg;
  return code;
}

int cuda_fail(cudaError_t e, const char* what) {
  g_last_error = std::string(what) + ": " + cudaGetErrorName(e) + " (" + cudaGetErrorString(e) + ")";
  return HIGGS_ERR_CUDA;
}

void qgemv_set_f16(bool on);
void attention_set_min_pages(int n);
void set_l2_prefetch(int mode);
void set_gemm_tc(bool on);
void set_gemm_tc_rows(int m);
void set_gemm_tc_waves(int w);
void set_gemm_tc_wave_cost(int c);
void qgemv_set_wk(int wk);
void qgemv_set_xsmem_max(int bytes);
void qgemv_m1_set(int on, int wk, int depth, int l2, int persist, int l1);
void qgemm_tc_prepare();
void decode_chain_set(int on, int l2_ahead);
void qgemv_tma_set(int on);
void attention_set_cluster(int n);
void model_set_tp_fuse(int on);
void attention_set_tq4_p_lo(int on);
void attention_set_tq4_swap(int n);
void prefill_attn_tc_set(int on);

}  // namespace higgs

using namespace higgs;

extern "C" int higgs_set_option(const char* name, int value) {
  HG_CHECK_ARG(name, "higgs_set_option: null name");
  const std::string n(name);
  if (n == "gemv_f16") {
    qgemv_set_f16(value != 0);
    return HIGGS_OK;
  }
  if (n == "gemv_xsmem_max") {
    qgemv_set_xsmem_max(value);
    return HIGGS_OK;
  }
  if (n == "gemv_wk") {
    qgemv_set_wk(value);
    return HIGGS_OK;
  }
  if (n == "gemv_m1") {
    qgemv_m1_set(value != 0, -1, -1, -1, -1, -1);
    return HIGGS_OK;
  }
  if (n == "gemv_m1_wk") {
    qgemv_m1_set(-1, value, -1, -1, -1, -1);
    return HIGGS_OK;
  }
  if (n == "gemv_m1_depth") {
    qgemv_m1_set(-1, -1, value, -1, -1, -1);
    return HIGGS_OK;
  }
  if (n == "gemv_m1_persist") {
    qgemv_m1_set(-1, -1, -1, -1, value, -1);
    return HIGGS_OK;
  }
  if (n == "gemv_m1_l1") {
    qgemv_m1_set(-1, -1, -1, -1, -1, value);
    return HIGGS_OK;
  }
  if (n == "attn_prefill_tc") {
    prefill_attn_tc_set(value);
    return HIGGS_OK;
  }
  if (n == "tq4_swap") {
    attention_set_tq4_swap(value);
    return HIGGS_OK;
  }
  if (n == "tq4_p_lo") {
    attention_set_tq4_p_lo(value);
    return HIGGS_OK;
  }
  if (n == "tp_fuse") {
    model_set_tp_fuse(value);
    return HIGGS_OK;
  }
  if (n == "attn_cluster") {
    attention_set_cluster(value);
    return HIGGS_OK;
  }
  if (n == "gemv_tma") {
    qgemv_tma_set(value != 0);
    return HIGGS_OK;
  }
  if (n == "decode_chain") {
    decode_chain_set(value != 0, -1);
    return HIGGS_OK;
  }
  if (n == "decode_chain_l2_ahead") {
    decode_chain_set(-1, value != 0);
    return HIGGS_OK;
  }
  if (n == "gemv_m1_l2") {
    qgemv_m1_set(-1, -1, -1, value, -1, -1);
    return HIGGS_OK;
  }
  if (n == "gemm_tc_rows") {
    set_gemm_tc_rows(value);
    return HIGGS_OK;
  }
  if (n == "gemm_tc_waves") {
    set_gemm_tc_waves(value);
    return HIGGS_OK;
  }
  if (n == "gemm_tc_wave_cost") {
    set_gemm_tc_wave_cost(value);
    return HIGGS_OK;
  }
  if (n == "gemm_tc") {
    set_gemm_tc(value != 0);
    return HIGGS_OK;
  }
  if (n == "l2_prefetch") {
    set_l2_prefetch(value);
    return HIGGS_OK;
  }
  if (n == "attn_min_pages") {
    attention_set_min_pages(value);
    return HIGGS_OK;
  }
  return fail(HIGGS_ERR_INVALID_ARG, "higgs_set_option: unknown option '" + n + "'");
}

extern "C" int higgs_version(void) { return 1; }

extern "C" const char* higgs_last_error(void) { return g_last_error.c_str(); }

extern "C" int higgs_init(int device, higgs_ctx** out) {
  HG_CHECK_ARG(out != nullptr, "higgs_init: out is null");
  *out = nullptr;
  int n = 0;
  HG_CUDA(cudaGetDeviceCount(&n));
  HG_CHECK_ARG(device >= 0 && device < n, "higgs_init: no such device");
  HG_CHECK_ARG(device < kMaxDevices, "higgs_init: device ordinal above 63");
  DeviceGuard guard;  // set-up runs on `device`; the caller's current device is restored
  if (int e = guard.enter(device)) return e;
  int major = 0, minor = 0, sms = 0;
  HG_CUDA(cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, device));
  HG_CUDA(cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, device));
  HG_CUDA(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device));
  if (major != 10 || minor != 0)
    return fail(HIGGS_ERR_UNSUPPORTED, "higgs_init: device is sm_" + std::to_string(major) +
                                           std::to_string(minor) + ", this build targets sm_100a");
  if (int e = device_setup(device, sms)) return e;
  qgemm_tc_prepare();
  higgs_ctx* c = new higgs_ctx;
  c->device = device;
  c->sms = sms;
  *out = c;
  return HIGGS_OK;
}

extern "C" int higgs_destroy(higgs_ctx* ctx) {
  delete ctx;
  return HIGGS_OK;
}
