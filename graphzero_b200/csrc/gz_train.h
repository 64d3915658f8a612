// Training steps of the GAT (train.cu) and the Connect4 ResNet
// (train_resnet.cu): buffers, kernels' host launchers, and the per-net
// training state (Adam moments, activations kept for the backward pass).
// Internal to the library; the C ABI is in graphzero_b200.h.
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

#include <functional>

namespace gz {
namespace train {

// Floats of the column-sum scratch: 64 row slices of up to 4672 columns.
constexpr size_t kColsumFloats = (size_t)64 * 4672;

// Scratch shared by the GEMMs (split-K partials) and the column sums.
struct Workspace {
  float* split = nullptr;
  size_t split_floats = 0;
  float* colsum = nullptr;  // [64 slices][up to 4672 columns]
};

// Everything the training step of one net keeps on its device.
struct State {
  int kind = 0;                 // 0 = GAT, 1 = ResNet (the net kinds of graphzero_b200.h)
  int game = -1;
  int capacity = 0;             // positions the activation buffers hold
  size_t weight_count = 0;
  float* m = nullptr;           // Adam first moments (weight layout)
  float* v = nullptr;           // Adam second moments
  float* grad = nullptr;        // gradient of the last step (weight layout)
  float* loss = nullptr;        // [2]: mean policy cross-entropy, mean value squared error
  int64_t step = 0;             // Adam steps taken
  int* graph = nullptr;         // row_ptr[N+1] | col[nnz] | rev[nnz]
  Workspace ws;
  float* arena = nullptr;       // activation and gradient buffers (see train.cu: layout())
  size_t arena_floats = 0;
  cudaStream_t comm_stream = nullptr;  // gradient all-reduce, beside the compute stream
  cudaEvent_t ev_bucket[16] = {};      // per bucket: its gradients are complete
  cudaEvent_t ev_comm = nullptr;       // all buckets reduced
};

// Adam hyper-parameters and bias-correction step.
struct AdamParams {
  float lr, beta1, beta2, eps, weight_decay, grad_scale;
};

// im2col 1 (2): A (B) is the 3 x 3 im2col matrix, [rows][9 * 128], of the
// [rows][128] Connect4 activation it points at, read in place (lda / ldb
// unused); needs gemm_big(M, N) and that operand untransposed.
cudaError_t gemm(Workspace& ws, int M, int N, int K, const float* A, int lda, bool ta, const float* B, int ldb,
                 bool tb, float* C, int ldc, bool accumulate, cudaStream_t s, int im2col = 0);
bool gemm_big(int M, int N);  // outputs that take the 128 x 128 tile kernel
cudaError_t colsum(Workspace& ws, const float* in, int R, int C, int ld, float* out, bool accumulate,
                   cudaStream_t s, float scale = 1.f);

// Allocates (or grows) the state for `game` and batches of up to
// `capacity` positions.  Returns a CUDA error on allocation failure.
cudaError_t ensure_state(State& st, int game, int capacity);
void free_state(State& st);

// One forward + backward pass over B positions (device int8 boards [B][board
// bytes], side [B], target policies [B][A], target values [B]) with the fp32
// weights `w`: the gradient of the mean loss lands in st.grad, the two loss
// terms in st.loss.  `bucket_done(k)` is called (on the host, in launch
// order) once the gradients of bucket k are complete on `s`: buckets
// 0 .. L-1 are the layers (W_l, b_l, a_l, contiguous in the layout), bucket L
// the heads.
cudaError_t loss_and_grad(State& st, const float* w, const int8_t* boards, const int8_t* side, const float* pi,
                          const float* v, int B, cudaStream_t s, const std::function<cudaError_t(int)>& bucket_done);

// w -= Adam(grad * grad_scale + weight_decay * w), step st.step + 1.
cudaError_t adam_step(State& st, float* w, const AdamParams& p, cudaStream_t s);

// Offset and length (floats) of gradient bucket k of `game`'s weight layout.
void bucket_range(int game, int k, size_t* offset, size_t* count);
int bucket_count(int game);

// The same for the Connect4 ResNet (res_layout weights).  Buckets: 0 the
// heads, 1 .. 10 the residual blocks from the last down, 11 the stem; BN
// means and variances are fixed (zero gradient, not updated by Adam).
cudaError_t res_ensure_state(State& st, int capacity);
cudaError_t res_loss_and_grad(State& st, const float* w, const int8_t* boards, const int8_t* side, const float* pi,
                              const float* v, int B, cudaStream_t s,
                              const std::function<cudaError_t(int)>& bucket_done);
cudaError_t res_adam_step(State& st, float* w, const AdamParams& p, cudaStream_t s);
void res_bucket_range(int k, size_t* offset, size_t* count);
constexpr int kResBuckets = 12;

}  // namespace train
}  // namespace gz
