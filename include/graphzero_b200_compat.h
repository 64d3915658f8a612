/*
 * Drop-in shim for GraphZero's model and game interfaces.
 *
 * The struct layouts mirror the reference's vtables so code written against
 * them (self_play/self_play.cu, arena/arena.cu, players/players.cu) binds
 * unchanged:
 *   INeuralNet      networks/neural_network.h:16-27
 *   TrainingExample networks/neural_network.h:10-14
 *   IGame           games/game.cuh:12-28
 * ncclComm_t and cudaStream_t appear as void* (same size, same calling
 * convention), so this header needs neither nccl.h nor the CUDA headers.
 * The functions behind the pointers call the gz_* C ABI
 * (graphzero_b200.h); the reference's versions return void and exit on
 * error, these return void too and report failures through gz_last_error().
 */
#ifndef GRAPHZERO_B200_COMPAT_H
#define GRAPHZERO_B200_COMPAT_H

#include <stdbool.h>

#include "graphzero_b200.h"

#ifdef __cplusplus
extern "C" {
#endif

#define GZ_MAX_BOARD_SIZE 64 /* MAX_BOARD_SIZE, games/game.cuh:7 */

typedef struct IGame IGame;
struct IGame {
  void (*init)(IGame* self);
  void (*get_init_board)(const IGame* self, int* board);
  void (*get_board_size)(const IGame* self, int* rows, int* cols);
  int (*get_action_size)(const IGame* self);
  void (*get_next_state)(const IGame* self, const int* board, int player, int action, int* next_board,
                         int* next_player);
  void (*get_valid_moves)(const IGame* self, const int* board, int player, bool* valid_moves);
  int (*get_game_ended)(const IGame* self, const int* board, int player);
  void (*get_canonical_form)(const IGame* self, const int* board, int player, int* canonical_board);
  float (*evaluate)(const IGame* self, const int* board, int player);
  void (*get_symmetries)(const IGame* self, const int* board, const float* pi, int (*symmetries)[GZ_MAX_BOARD_SIZE],
                         float (*symmetries_pi)[GZ_MAX_BOARD_SIZE], int* num_symmetries);
  void (*string_representation)(const IGame* self, const int* board, char* str, int str_size);
  void (*display)(const IGame* self, const int* board);
};

typedef struct {
  float* board;
  float* pi;
  float v;
} TrainingExample;

typedef struct INeuralNet INeuralNet;
struct INeuralNet {
  void* impl;
  void (*init)(INeuralNet* self, const IGame* game);
  void (*train)(INeuralNet* self, TrainingExample* examples, int num_examples);
  void (*predict)(INeuralNet* self, const float* board, float* pi, float* v);
  void (*save_checkpoint)(INeuralNet* self, const char* folder, const char* filename);
  void (*load_checkpoint)(INeuralNet* self, const char* folder, const char* filename);
  void (*destroy)(INeuralNet* self);
  void (*train_distributed)(INeuralNet* self, float* d_boards, float* d_pis, float* d_vs, int num_examples,
                            int world_rank, int world_size, void* nccl_comm, void* cuda_stream);
  void (*broadcast_weights)(INeuralNet* self, int world_rank, int world_size, void* nccl_comm, void* cuda_stream);
};

/* Game factories (games/connect4/connect4.cu:140-167 create_connect4_game,
 * games/tictactoe/tictactoe.cu:166-194 create_tictactoe_game).  Release with
 * gz_game_free.  get_game_ended returns 1 / -1 for a win of `player` / of the
 * opponent and 0 otherwise; a draw also returns 0, as the reference's int
 * return type truncates its draw marker (connect4.cu:86). */
IGame* gz_create_connect4_game(void);
IGame* gz_create_tictactoe_game(void);
void gz_game_free(IGame* game);

/* create_neural_net(type, game) (networks/neural_network.c:6-13): "gat" or
 * "resnet" for the game's board size, on CUDA device `device`, weights from
 * the seeded Glorot generator (load a checkpoint to replace them).  NULL on
 * failure (see gz_last_error()). */
INeuralNet* gz_create_neural_net(const char* net_type, const IGame* game, int device);
/* The gz_net behind an INeuralNet made by gz_create_neural_net. */
gz_net* gz_shim_net(INeuralNet* nn);
/* Wraps an existing gz_net (not owned: destroy frees only the wrapper). */
INeuralNet* gz_shim_make_ineuralnet(gz_net* net);

#ifdef __cplusplus
}
#endif

#endif /* GRAPHZERO_B200_COMPAT_H */
