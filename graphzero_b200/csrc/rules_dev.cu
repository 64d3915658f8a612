// Game rules on the device: the seeded position generator for every game and
// chess legal-move generation in the reference's action indices, one thread
// per position.  Both run the same host/device functions as the host entry
// points (gz_games.h, gz_synth.h, gz_chess.h), so a position or a move list
// made here is byte-for-byte the one the host makes.
//
// Reference counterparts: games/connect4/connect4.cu:22-93,
// games/tictactoe/tictactoe.cu:24-72 (rules), games/chess/chess.cu:102-326
// and 677-1071 (chess rules and move generation; the latter does not
// compile, this is a standard legal generator).
#include <cuda_runtime.h>
#include <stdint.h>

#include "gz_chess.h"
#include "gz_games.h"
#include "gz_synth.h"

namespace gz {
namespace {

constexpr int kRulesThreads = 128;

__global__ void synth_positions_kernel(int game, uint64_t seed, uint64_t first, int n, int board_bytes,
                                       int8_t* __restrict__ boards, int8_t* __restrict__ side) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  int8_t* rec = boards + (size_t)i * board_bytes;  // written in place
  side[i] = (int8_t)(game == kChess ? chess::make_position(seed, first + (uint64_t)i, rec)
                                    : make_position(game, seed, first + (uint64_t)i, rec));
}

// Per position: the number of legal moves and their action indices in the
// generator's order; actions[i][count..255] are set to -1.
__global__ void chess_legal_kernel(const int8_t* __restrict__ boards, const int8_t* __restrict__ side, int n,
                                   int16_t* __restrict__ actions, int32_t* __restrict__ counts) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  chess::Pos p;
  chess::from_record(boards + (size_t)i * 66, side[i], p);
  chess::Move ms[256];
  const int c = chess::legal_moves_inplace(p, ms);
  int16_t* out = actions + (size_t)i * 256;
  for (int k = 0; k < 256; ++k) out[k] = k < c ? (int16_t)chess::encode_action(ms[k]) : (int16_t)-1;
  counts[i] = c;
}

}  // namespace

cudaError_t launch_synth_positions(int game, uint64_t seed, uint64_t first, int n, int8_t* boards, int8_t* side,
                                   cudaStream_t stream) {
  if (n <= 0) return cudaSuccess;
  const GameShape s = game_shape(game);
  synth_positions_kernel<<<(n + kRulesThreads - 1) / kRulesThreads, kRulesThreads, 0, stream>>>(
      game, seed, first, n, s.board_bytes, boards, side);
  return cudaGetLastError();
}

cudaError_t launch_chess_legal(const int8_t* boards, const int8_t* side, int n, int16_t* actions, int32_t* counts,
                               cudaStream_t stream) {
  if (n <= 0) return cudaSuccess;
  chess_legal_kernel<<<(n + kRulesThreads - 1) / kRulesThreads, kRulesThreads, 0, stream>>>(boards, side, n, actions,
                                                                                             counts);
  return cudaGetLastError();
}

}  // namespace gz
