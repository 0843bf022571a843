// Error plumbing, status strings and host-side random draws.
#include <cmath>
#include <cstdio>
#include <random>
#include <string>

#include "common.cuh"

namespace dcc {

static thread_local std::string g_last_error;

void set_error(const std::string& msg) { g_last_error = msg; }

int fail(int status, const std::string& msg) {
  g_last_error = msg;
  return status;
}

int check_cuda(cudaError_t e, const char* what) {
  if (e == cudaSuccess) return DCC_OK;
  return fail(DCC_ERR_CUDA, std::string(what) + ": " + cudaGetErrorString(e));
}

int check_launch(const char* what) { return check_cuda(cudaGetLastError(), what); }

int num_sms() {
  int dev = 0, n = 148;
  if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
  return n > 0 ? n : 148;
}

}  // namespace dcc

extern "C" {

const char* dcc_status_string(int status) {
  switch (status) {
    case DCC_OK: return "ok";
    case DCC_ERR_INVALID_ARGUMENT: return "invalid argument";
    case DCC_ERR_SHAPE: return "shape mismatch";
    case DCC_ERR_DTYPE: return "unsupported dtype";
    case DCC_ERR_WORKSPACE: return "workspace too small";
    case DCC_ERR_CUDA: return "CUDA error";
    case DCC_ERR_UNSUPPORTED: return "unsupported size";
    case DCC_ERR_TIMEOUT: return "device wait timed out";
    default: return "unknown status";
  }
}

const char* dcc_last_error(void) { return dcc::g_last_error.c_str(); }

int dcc_version(void) { return 2; }

size_t dcc_struct_size(const char* name) {
  if (!name) return 0;
  const std::string n(name);
  if (n == "dcc_query_set") return sizeof(dcc_query_set);
  if (n == "dcc_build_problem") return sizeof(dcc_build_problem);
  if (n == "dcc_kv_segment") return sizeof(dcc_kv_segment);
  if (n == "dcc_attn_problem") return sizeof(dcc_attn_problem);
  return 0;
}

// torch's CPU generator is mt19937 seeded with the low 32 bits of the seed
// (the standard init_genrand); randint(lo, hi) for a range below 2^32 is
// lo + raw32 % (hi - lo), filled in element order.  std::mt19937 is the same
// engine with the same seeding.
int dcc_rademacher_projection(int head_dim, int projection_dim, uint64_t seed, float* out_host) {
  if (head_dim <= 0 || projection_dim <= 0 || out_host == nullptr)
    return dcc::fail(DCC_ERR_INVALID_ARGUMENT, "rademacher_projection: bad arguments");
  std::mt19937 eng(static_cast<uint32_t>(seed & 0xFFFFFFFFu));
  const float denom = static_cast<float>(std::sqrt(static_cast<double>(projection_dim)));
  for (int i = 0; i < projection_dim * head_dim; ++i) {
    const uint32_t r = eng();
    const float sign = (r % 2u) ? 1.0f : -1.0f;
    out_host[i] = sign / denom;
  }
  return DCC_OK;
}

int64_t dcc_fps_start_index(int64_t num_points, uint64_t seed) {
  if (num_points <= 0) return -1;
  std::mt19937 eng(static_cast<uint32_t>(seed & 0xFFFFFFFFu));
  return static_cast<int64_t>(static_cast<uint64_t>(eng()) % static_cast<uint64_t>(num_points));
}

}  // extern "C"
