// Process-wide device status word used by bounded waits in every pipelined kernel.
#include "common.cuh"

namespace tdsv {

namespace {
__device__ int g_status_word;
constexpr int kMaxDevices = 64;
int* g_status_ptr[kMaxDevices] = {nullptr};
// How long a wait on another rank's flag may spin before it records kTimeoutPeer and returns.
uint64_t g_peer_wait_limit_ns = kWaitLimitNs;
}  // namespace

uint64_t peer_wait_limit_ns() { return g_peer_wait_limit_ns; }

void set_peer_wait_limit_ns(int64_t ns) {
  TDSV_CHECK(ns > 0, "set_peer_wait_limit_ns: the limit must be positive");
  g_peer_wait_limit_ns = static_cast<uint64_t>(ns);
}

// The status word of the current device as a one-element int32 CUDA tensor that aliases it (no
// ownership), so the host can snapshot it asynchronously into pinned memory once per step.
at::Tensor status_word() {
  int dev = 0;
  TDSV_CUDA_CHECK(cudaGetDevice(&dev));
  return at::from_blob(status_word_ptr(), {1}, at::TensorOptions().dtype(at::kInt).device(at::kCUDA, dev));
}

int* status_word_ptr() {
  int dev = 0;
  TDSV_CUDA_CHECK(cudaGetDevice(&dev));
  TDSV_CHECK(dev < kMaxDevices, "device index out of range");
  if (g_status_ptr[dev] == nullptr) {
    void* p = nullptr;
    TDSV_CUDA_CHECK(cudaGetSymbolAddress(&p, g_status_word));
    g_status_ptr[dev] = static_cast<int*>(p);
  }
  return g_status_ptr[dev];
}

// Reads the status word on the current stream (synchronising it), resets it and raises.
void check_status(const char* what) {
  int host = 0;
  int* dptr = status_word_ptr();
  cudaStream_t s = stream();
  TDSV_CUDA_CHECK(cudaMemcpyAsync(&host, dptr, sizeof(int), cudaMemcpyDeviceToHost, s));
  TDSV_CUDA_CHECK(cudaStreamSynchronize(s));
  if (host != 0) {
    int zero = 0;
    TDSV_CUDA_CHECK(cudaMemcpyAsync(dptr, &zero, sizeof(int), cudaMemcpyHostToDevice, s));
    TDSV_CUDA_CHECK(cudaStreamSynchronize(s));
    TORCH_CHECK(false, what, ": device pipeline reported status ", host,
                " (1/2 = TMA stage wait timed out, 3/4 = accumulator wait timed out, 5 = peer flag "
                "timed out, 6 = bad shape, 7 = index out of bounds (bounds-check build), 3xx / 4xx = "
                "attention / indexer pipeline wait timed out)");
  }
}

int64_t read_status() {
  int host = 0;
  int* dptr = status_word_ptr();
  cudaStream_t s = stream();
  TDSV_CUDA_CHECK(cudaMemcpyAsync(&host, dptr, sizeof(int), cudaMemcpyDeviceToHost, s));
  TDSV_CUDA_CHECK(cudaStreamSynchronize(s));
  int zero = 0;
  TDSV_CUDA_CHECK(cudaMemcpyAsync(dptr, &zero, sizeof(int), cudaMemcpyHostToDevice, s));
  TDSV_CUDA_CHECK(cudaStreamSynchronize(s));
  return host;
}

}  // namespace tdsv
