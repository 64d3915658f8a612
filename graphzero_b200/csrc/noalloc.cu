// Connect4 GAT leaf evaluation without any device allocation.
//
// For callers that are not allowed to allocate device memory: plugins that
// run inside a host application which owns the CUDA context and fixes the
// device-memory budget at start-up, and latency-critical loops that cannot
// afford cudaMalloc/cudaFree (they synchronise the device and take an
// unbounded time).  Such a caller has no gz_net handle (creating one
// allocates); it passes host weights, positions and output buffers, and this
// entry point stages everything through one file-scope device array:
//
//   fp32 weight blob | packed weight tiles | boards | side | pi | v | error word
//
// All of it is device memory reserved when the library is loaded, on every
// GPU the process uses, until the process exits.  Positions per call are
// limited to kNoAllocMaxBatch.  Every call shares the array and finds the
// previous call's contents in it: the weights, positions and the error word
// are rewritten on every call, so nothing carries over, but calls that
// overlap in time (two host threads, or two devices sharing nothing but this
// entry point) on the same device race on the array and must be serialised
// by the caller.
//
// Each call uploads the whole 1.4 MB fp32 weight blob and repacks it (one
// small kernel) before the forward pass, and runs on the device's legacy
// default stream, which also waits for the work of every blocking stream of
// the process on that device.  The kernel and operand format are those of a
// gz_net created with GZ_PREC_AUTO, so both give identical outputs.
//
// The array's device address is looked up on the first call on a device
// (cudaGetSymbolAddress with that device current) and kept per device
// together with the identity of the CUDA context it belongs to; after a
// cudaDeviceReset the next call finds a new context and looks the address up
// again.
#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>
#include <string.h>

#include <mutex>

#include "../../include/graphzero_b200.h"
#include "gz_games.h"
#include "gz_internal.h"

namespace gz {
namespace {

constexpr int kNoAllocMaxBatch = 4096;
constexpr int kC4Board = 42;
constexpr int kC4Actions = 7;

// Byte offsets inside the scratch array (each part 256-byte aligned).
constexpr size_t align256(size_t x) { return (x + 255) & ~(size_t)255; }
constexpr size_t kWeightsFloats = 350082;  // Connect4 GAT blob (gat_layout), checked at run time
constexpr size_t kOffWeights = 0;
constexpr size_t kOffPacked = align256(kOffWeights + kWeightsFloats * sizeof(float));
constexpr size_t kPackedBytes = 21 * 36864;  // checked against gat_tc_packed_bytes at run time
constexpr size_t kOffBoards = align256(kOffPacked + kPackedBytes);
constexpr size_t kOffSide = align256(kOffBoards + (size_t)kNoAllocMaxBatch * kC4Board);
constexpr size_t kOffPi = align256(kOffSide + kNoAllocMaxBatch);
constexpr size_t kOffV = align256(kOffPi + (size_t)kNoAllocMaxBatch * kC4Actions * sizeof(float));
constexpr size_t kOffErr = align256(kOffV + (size_t)kNoAllocMaxBatch * sizeof(float));
constexpr size_t kScratchBytes = align256(kOffErr + sizeof(int));

static __device__ __align__(256) uint8_t g_noalloc_scratch[kScratchBytes];

// Device address of g_noalloc_scratch per device, looked up on the first call
// on that device (with that device current), and the id of the context it
// was looked up in.
uint8_t* g_scratch_addr[64];
unsigned long long g_scratch_ctx[64];
std::mutex g_setup_mutex;

// Id of the calling thread's current CUDA context (unique over the process's
// lifetime), or 0 if the driver cannot tell; through the runtime's driver
// entry points, so the library needs no link to libcuda.
unsigned long long current_context_id() {
  using GetCurrent = CUresult (*)(CUcontext*);
  using GetId = CUresult (*)(CUcontext, unsigned long long*);
  static GetCurrent get_current = nullptr;
  static GetId get_id = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* f = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPointByVersion("cuCtxGetCurrent", &f, 12000, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      get_current = (GetCurrent)f;
    f = nullptr;
    if (cudaGetDriverEntryPointByVersion("cuCtxGetId", &f, 12000, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      get_id = (GetId)f;
    cudaGetLastError();
  });
  CUcontext ctx = nullptr;
  unsigned long long id = 0;
  if (!get_current || !get_id || get_current(&ctx) != CUDA_SUCCESS || !ctx || get_id(ctx, &id) != CUDA_SUCCESS) return 0;
  return id;
}

}  // namespace
}  // namespace gz

extern "C" {

size_t gz_gat_c4_noalloc_scratch_bytes(void) { return gz::kScratchBytes; }
int gz_gat_c4_noalloc_max_batch(void) { return gz::kNoAllocMaxBatch; }

gz_status gz_gat_c4_predict_noalloc(int device, const float* h_weights, size_t n_weights, const int8_t* h_boards,
                                    const int8_t* h_side, int n, float* h_pi, float* h_v) {
  using namespace gz;
  if (n < 0 || n > kNoAllocMaxBatch)
    return set_last_error(GZ_ERR_INVALID_ARG, "gz_gat_c4_predict_noalloc: batch of %d positions outside [0, %d] "
                                              "(the fixed device scratch holds at most %d)",
                          n, kNoAllocMaxBatch, kNoAllocMaxBatch);
  if (n_weights != kWeightsFloats || gat_layout(kConnect4).total != kWeightsFloats ||
      gat_tc_packed_bytes(kConnect4) != kPackedBytes)
    return set_last_error(GZ_ERR_INVALID_ARG, "gz_gat_c4_predict_noalloc: weight blob has %zu floats, the Connect4 "
                                              "GAT blob has %zu", n_weights, (size_t)kWeightsFloats);
  if (!h_weights || (n > 0 && (!h_boards || !h_side || !h_pi || !h_v)))
    return set_last_error(GZ_ERR_INVALID_ARG, "gz_gat_c4_predict_noalloc: null buffer");
  if (device < 0 || device >= 64) return set_last_error(GZ_ERR_INVALID_ARG, "bad device %d", device);
  int prev = -1;
  if (cudaGetDevice(&prev) != cudaSuccess || cudaSetDevice(device) != cudaSuccess)
    return set_last_error(GZ_ERR_CUDA, "cannot select CUDA device %d", device);
  gz_status st = GZ_OK;
  uint8_t* base = nullptr;
  {
    std::lock_guard<std::mutex> lock(g_setup_mutex);
    const unsigned long long ctx = current_context_id();
    if (!g_scratch_addr[device] || ctx == 0 || ctx != g_scratch_ctx[device]) {
      void* ptr = nullptr;
      const cudaError_t e = cudaGetSymbolAddress(&ptr, g_noalloc_scratch);
      g_scratch_addr[device] = nullptr;
      if (e != cudaSuccess || !ptr)
        st = set_last_error(GZ_ERR_CUDA, "cudaGetSymbolAddress of the scratch array: %s", cudaGetErrorString(e));
      else {
        g_scratch_addr[device] = (uint8_t*)ptr;
        g_scratch_ctx[device] = ctx;
      }
    }
    base = g_scratch_addr[device];
  }
  if (st == GZ_OK && n > 0) {
    float* d_w = (float*)(base + kOffWeights);
    uint8_t* d_packed = base + kOffPacked;
    int8_t* d_boards = (int8_t*)(base + kOffBoards);
    int8_t* d_side = (int8_t*)(base + kOffSide);
    float* d_pi = (float*)(base + kOffPi);
    float* d_v = (float*)(base + kOffV);
    int* d_err = (int*)(base + kOffErr);
    cudaStream_t s = 0;  // legacy default stream of the device: ordered with the copies below
    cudaError_t e = cudaMemcpyAsync(d_w, h_weights, n_weights * sizeof(float), cudaMemcpyHostToDevice, s);
    if (e == cudaSuccess) e = cudaMemcpyAsync(d_boards, h_boards, (size_t)n * kC4Board, cudaMemcpyHostToDevice, s);
    if (e == cudaSuccess) e = cudaMemcpyAsync(d_side, h_side, (size_t)n, cudaMemcpyHostToDevice, s);
    if (e == cudaSuccess) e = cudaMemsetAsync(d_err, 0, sizeof(int), s);  // the error word starts at zero
    if (e == cudaSuccess) e = launch_gat_tc_pack(kConnect4, kAutoFp16, d_w, d_packed, s);
    if (e == cudaSuccess) e = launch_gat_tc(kConnect4, kAutoFp16, d_packed, d_w, d_boards, d_side, n, d_pi, d_v, d_err, s);
    if (e == cudaSuccess) e = cudaMemcpyAsync(h_pi, d_pi, (size_t)n * kC4Actions * sizeof(float), cudaMemcpyDeviceToHost, s);
    if (e == cudaSuccess) e = cudaMemcpyAsync(h_v, d_v, (size_t)n * sizeof(float), cudaMemcpyDeviceToHost, s);
    int err = 0;
    if (e == cudaSuccess) e = cudaMemcpyAsync(&err, d_err, sizeof(int), cudaMemcpyDeviceToHost, s);
    if (e == cudaSuccess) e = cudaStreamSynchronize(s);
    if (e != cudaSuccess) st = set_last_error(GZ_ERR_CUDA, "gz_gat_c4_predict_noalloc: %s", cudaGetErrorString(e));
    else if (err) st = forward_error_status(err, "gz_gat_c4_predict_noalloc");
  }
  cudaSetDevice(prev);
  return st;
}

}  // extern "C"
