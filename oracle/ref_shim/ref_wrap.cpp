// C entry points over the reference's own rule functions (compiled unmodified
// from games/connect4/connect4.cu and games/tictactoe/tictactoe.cu).
// Test infrastructure only: tests compare the oracle's restated rules with
// these on many positions.
#include <stdint.h>
#include "game.h"

void connect4_get_next_state(const IGame*, const int*, int, int, int*, int*);
void connect4_get_valid_moves(const IGame*, const int*, int, bool*);
int connect4_get_game_ended(const IGame*, const int*, int);
void connect4_get_canonical_form(const IGame*, const int*, int, int*);
void tictactoe_get_next_state(const IGame*, const int*, int, int, int*, int*);
void tictactoe_get_valid_moves(const IGame*, const int*, int, bool*);
int tictactoe_get_game_ended(const IGame*, const int*, int);
void tictactoe_get_canonical_form(const IGame*, const int*, int, int*);

extern "C" {
// game: 0 = TicTacToe, 1 = Connect4
void ref_next_state(int game, const int* board, int player, int action, int* next_board, int* next_player) {
  if (game == 1) connect4_get_next_state(nullptr, board, player, action, next_board, next_player);
  else tictactoe_get_next_state(nullptr, board, player, action, next_board, next_player);
}
void ref_valid_moves(int game, const int* board, int player, uint8_t* valid) {
  bool v[64] = {false};
  if (game == 1) connect4_get_valid_moves(nullptr, board, player, v);
  else tictactoe_get_valid_moves(nullptr, board, player, v);
  int n = game == 1 ? 7 : 9;
  for (int i = 0; i < n; ++i) valid[i] = v[i] ? 1 : 0;
}
int ref_game_ended(int game, const int* board, int player) {
  return game == 1 ? connect4_get_game_ended(nullptr, board, player) : tictactoe_get_game_ended(nullptr, board, player);
}
void ref_canonical(int game, const int* board, int player, int* out) {
  if (game == 1) connect4_get_canonical_form(nullptr, board, player, out);
  else tictactoe_get_canonical_form(nullptr, board, player, out);
}
}
