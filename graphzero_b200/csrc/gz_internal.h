// Internal declarations shared by the graphzero_b200 CUDA translation units.
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

#include "gz_games.h"

#include "../../include/graphzero_b200.h"

namespace gz {

// Records a printf-style message for gz_last_error() of the calling thread
// and returns `s`.
gz_status set_last_error(gz_status s, const char* fmt, ...);

// The operand format GZ_PREC_AUTO picks for the tensor-core kernels: fp16
// (11 significant bits, the same tensor-core rate as bf16).  Its rounding
// error is 6-8x smaller than bf16's on these networks; activations must stay
// below 65504 in magnitude (GZ_PREC_BF16 has the fp32 range).
constexpr bool kAutoFp16 = true;

// Status of a forward kernel's error word: 0 ok, 2 the dynamic shared
// memory base was not 1024-byte aligned (GZ_ERR_CUDA), anything else a
// bounded wait that gave up (GZ_ERR_TIMEOUT).  `who` prefixes the message.
gz_status forward_error_status(int err, const char* who);

// Game of a net (for the INeuralNet shim).
int net_game(const gz_net* net);
// ncclBroadcast of `count` floats from `root`, in place (NCCL loaded at run
// time); for the INeuralNet shim's train_distributed.
gz_status nccl_broadcast_floats(void* comm, float* d_buf, size_t count, int root, void* stream);

// fp32 SIMT fused GAT forward (all layers + heads, one launch).
//   boards [n][BOARD] int8, side [n] int8 (+1 / -1),
//   weights: fp32 blob in gat_layout() order,
//   csr: row_ptr [N+1] followed by col [nnz] (build_graph_csr order),
//   pi [n][A] fp32, v [n] fp32.
cudaError_t launch_gat_simt(int game, const float* d_weights, const int* d_csr, const int8_t* d_boards,
                            const int8_t* d_side, int n, float* d_pi, float* d_v, cudaStream_t stream);
// The same for TicTacToe, laid out for its 9-node stencil graph (gat_simt_ttt.cu).
cudaError_t launch_gat_simt_ttt(const float* d_weights, const int8_t* d_boards, const int8_t* d_side, int n,
                                float* d_pi, float* d_v, cudaStream_t stream);

// Tensor-core (tcgen05) GAT forward for Connect4 and chess, bf16 or fp16 operands.
// gat_tc_packed_bytes(game) is 0 when the game has no tensor-core kernel.
size_t gat_tc_packed_bytes(int game);
// Converts the fp32 blob into the kernel's operand layout (bf16 or fp16
// weight tiles, 128-byte swizzled).
cudaError_t launch_gat_tc_pack(int game, int fp16, const float* d_weights, void* d_packed, cudaStream_t stream);
// d_err: device word set to 1 when a bounded wait inside the kernel gave up.
cudaError_t launch_gat_tc(int game, int fp16, const void* d_packed, const float* d_weights, const int8_t* d_boards,
                          const int8_t* d_side, int n, float* d_pi, float* d_v, int* d_err, cudaStream_t stream);

// Chess tensor-core GAT (gat_tc_chess.cu); reached through the gat_tc
// functions above with game == chess.
size_t chess_tc_packed_bytes();
cudaError_t launch_chess_tc_pack(int fp16, const float* d_weights, void* d_packed, cudaStream_t stream);
cudaError_t launch_chess_tc(int fp16, const void* d_packed, const float* d_weights, const int8_t* d_boards,
                            const int8_t* d_side, int n, float* d_pi, float* d_v, int* d_err, cudaStream_t stream);

// Tensor-core Connect4 ResNet forward (implicit-GEMM 3x3 convolutions), bf16 or fp16 operands.
// rules_dev.cu: seeded positions on the device (bytes as gz_synth_positions
// makes them) and chess legal moves as action indices ([n][256], -1 padded).
cudaError_t launch_synth_positions(int game, uint64_t seed, uint64_t first, int n, int8_t* boards, int8_t* side,
                                   cudaStream_t stream);
cudaError_t launch_chess_legal(const int8_t* boards, const int8_t* side, int n, int16_t* actions, int32_t* counts,
                               cudaStream_t stream);

size_t resnet_tc_packed_bytes();
cudaError_t launch_resnet_tc_pack(int fp16, const float* d_weights, void* d_packed, cudaStream_t stream);
cudaError_t launch_resnet_tc(int fp16, const void* d_packed, const float* d_weights, const int8_t* d_boards,
                             const int8_t* d_side, int n, float* d_pi, float* d_v, int* d_err, cudaStream_t stream);

}  // namespace gz
