// Host-side helpers shared by every entry point: error text, launch checks,
// SM count, ABI version.
#include <math.h>
#include <stdio.h>

#include "common.cuh"

namespace nqt {

static thread_local char g_last_error[256] = "";

void set_last_error(const char* what, cudaError_t err) {
  snprintf(g_last_error, sizeof(g_last_error), "%s: %s", what, cudaGetErrorString(err));
}

void set_last_message(const char* what) { snprintf(g_last_error, sizeof(g_last_error), "%s", what); }

int check_launch(const char* what) {
  cudaError_t err = cudaGetLastError();
  if (err != cudaSuccess) {
    set_last_error(what, err);
    return NQT_ERR_CUDA;
  }
  return NQT_OK;
}

int num_sms() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return 148;
  int sms = 0;
  if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || sms <= 0) return 148;
  return sms;
}

void rope_inv_freq_table(float* out, int head_dim, float rope_theta) {
  const double ln_theta = log(static_cast<double>(rope_theta));
  for (int i = 0; i < head_dim / 2; ++i) out[i] = static_cast<float>(exp(-ln_theta * (2.0 * i / head_dim)));
}

}  // namespace nqt

extern "C" int nqt_abi_version(void) { return 1; }

extern "C" const char* nqt_last_error(void) { return nqt::g_last_error; }
