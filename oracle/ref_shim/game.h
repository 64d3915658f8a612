/* Stand-in for the reference's missing games/game.h (connect4.cuh:4 and
 * tictactoe.cuh:4 include "../game.h", which the reference does not ship).
 * It declares the IGame members that the reference's factories assign
 * (connect4.cu:140-167, tictactoe.cu:166-194): the games/game.cuh:12-28
 * vtable plus the *_cuda duplicates.  Test infrastructure only: used to compile
 * the reference's rule functions into oracle/_ref so the oracle's restated
 * rules can be checked against them. */
#ifndef GZ_REF_SHIM_GAME_H
#define GZ_REF_SHIM_GAME_H
#include <stdbool.h>
#include <stdlib.h>
#include <string.h>
#define __host__
#define __device__
#define MAX_BOARD_SIZE 64
typedef struct IGame IGame;
struct IGame {
  void (*init)(IGame*);
  void (*get_init_board)(const IGame*, int*);
  void (*get_board_size)(const IGame*, int*, int*);
  int (*get_action_size)(const IGame*);
  void (*get_next_state)(const IGame*, const int*, int, int, int*, int*);
  void (*get_valid_moves)(const IGame*, const int*, int, bool*);
  int (*get_game_ended)(const IGame*, const int*, int);
  void (*get_canonical_form)(const IGame*, const int*, int, int*);
  float (*evaluate)(const IGame*, const int*, int);
  void (*get_symmetries)(const IGame*, const int*, const float*, int (*)[MAX_BOARD_SIZE], float (*)[MAX_BOARD_SIZE], int*);
  void (*string_representation)(const IGame*, const int*, char*, int);
  void (*display)(const IGame*, const int*);
  void (*get_init_board_cuda)(const IGame*, int*);
  void (*get_next_state_cuda)(const IGame*, const int*, int, int, int*, int*);
  void (*get_valid_moves_cuda)(const IGame*, const int*, int, bool*);
  int (*get_game_ended_cuda)(const IGame*, const int*, int);
  void (*get_canonical_form_cuda)(const IGame*, const int*, int, int*);
  float (*evaluate_cuda)(const IGame*, const int*, int);
};
#endif
