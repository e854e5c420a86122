// C-ABI plumbing: error messages, ABI version, capability query and the
// device error word.
#include <cstdarg>
#include <cstring>

#include "common.cuh"

namespace kf {

namespace {
thread_local char g_msg[1024] = "";
}

namespace {
DeviceErrorReader g_readers[32];
int g_n_readers = 0;
}  // namespace

void register_device_error_reader(DeviceErrorReader fn) {
  // called from static initialisers of each translation unit, before main
  if (g_n_readers < 32) g_readers[g_n_readers++] = fn;
}

void set_error(const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_msg, sizeof(g_msg), fmt, ap);
  va_end(ap);
}

void clear_error() { g_msg[0] = '\0'; }

int check_launch(const char* what) {
  cudaError_t err = cudaGetLastError();
  if (err != cudaSuccess) {
    set_error("%s: launch failed: %s", what, cudaGetErrorString(err));
    return KF_ERR_CUDA;
  }
  return KF_OK;
}

}  // namespace kf

int kf::bind_device(const void* ptr) {
  cudaPointerAttributes attr;
  cudaError_t err = cudaPointerGetAttributes(&attr, ptr);
  if (err != cudaSuccess || (attr.type != cudaMemoryTypeDevice && attr.type != cudaMemoryTypeManaged)) {
    cudaGetLastError();
    set_error("operand %p is not CUDA device memory", ptr);
    return KF_ERR_ARG;
  }
  // Since CUDA 12, cudaSetDevice initialises the device's primary context and
  // makes it current on this thread immediately, which the driver calls of
  // the tensor-map encoder need.
  KF_CUDA_RET(cudaSetDevice(attr.device));
  return KF_OK;
}

extern "C" int kf_version(void) { return KF_ABI_VERSION; }

extern "C" const char* kf_last_error(void) { return kf::g_msg; }

extern "C" int kf_device_status(int32_t* flags) {
  using namespace kf;
  clear_error();
  KF_CHECK_ARG(flags != nullptr, "kf_device_status: flags is null");
  KF_CUDA_RET(cudaDeviceSynchronize());
  int32_t v = 0;
  for (int r = 0; r < g_n_readers; ++r) {
    if (g_readers[r](&v) != KF_OK) {
      set_error("kf_device_status: reading the device error word failed: %s", cudaGetErrorString(cudaGetLastError()));
      return KF_ERR_CUDA;
    }
  }
  *flags = v;
  return KF_OK;
}

// Fused tensor-core kernels: the feature vector of one input (basis features
// plus the SiLU column) must fit the padded width; B-splines up to order 5.
static int closed_family_ok(const kf_basis_desc* d) {
  if (d->kind == KF_BASIS_FOURIER) return d->size >= 2 && d->size % 2 == 0 && d->size <= 32 && d->period > 0.0f;
  if (d->kind == KF_BASIS_BUMP)
    return d->size >= 2 && d->size <= 32 && (d->bump_mode == KF_BUMP_GAUSS || d->bump_mode == KF_BUMP_TANH);
  return 0;
}

static int fused_supported(const kf_basis_desc* d) {
  if (d->kind == KF_BASIS_CHEB) return d->degree + 2 <= 32;
  if (d->kind == KF_BASIS_FOURIER) return closed_family_ok(d) && d->size + 1 <= 32;
  if (d->kind == KF_BASIS_BSPLINE) return d->order >= 1 && d->order <= 5 && d->size + 1 <= 32 && d->grid_size + 2 * d->order + 1 <= 64;
  return 0;
}

extern "C" int kf_query(const kf_basis_desc* d, int op, int dtype) {
  if (d == nullptr) return 0;
  switch (op) {
    case KF_OP_F:
    case KF_OP_G:
    case KF_OP_P:
      if (dtype != KF_DTYPE_F32) return 0;
      if (d->kind == KF_BASIS_CHEB) return d->degree + 1 <= 32;
      if (d->kind == KF_BASIS_BSPLINE)
        return d->order >= 1 && d->order <= 5 && d->size <= 32 && d->grid_size + 2 * d->order + 1 <= 64;
      return closed_family_ok(d);
    case 16:
      return dtype == KF_DTYPE_BF16 && fused_supported(d);
    case 17:
      if (dtype != KF_DTYPE_F32) return 0;
      if (d->kind == KF_BASIS_RATIONAL) return d->degree + 1 <= 12 && d->den_degree <= 12;
      if (d->kind == KF_BASIS_CHEB) return d->degree + 1 <= 32;
      if (d->kind == KF_BASIS_BSPLINE)
        return d->order >= 1 && d->order <= 5 && d->size <= 32 && d->grid_size + 2 * d->order + 1 <= 64;
      return closed_family_ok(d);
    default:
      return 0;
  }
}
