"""Sequential CPU restatement of the batched PUCT waves on chess
(test infrastructure).

It repeats, tree by tree and leaf by leaf, what the search kernels do for
chess (graphzero_b200/csrc/mcts.cu, chess_*): `leaves` selections per tree
with virtual loss, the PUCT score in float32 with the kernels' operation
order, the lowest edge index on ties, a new node checked for checkmate
(a loss for its player to move) or stalemate (a draw), expansion with the
policy renormalised over the leaf's legal actions in generation order, and
the backup with the value's sign flipping every level.  Reference
semantics: self_play/self_play.cu:720-758 (PUCT, backup), 698-718
(expansion), mcts/mcts.cu:68-103 (re-rooting).

The chess rules come from the library's host entry points
(gz.chess_legal_actions / chess_next_state / chess_ended), which the perft
known-answer tests pin on their own (tests/test_chess_rules.py); what this
module restates is the search.
"""
from __future__ import annotations

import numpy as np

import graphzero_b200 as gz

F = np.float32
MAX_DEPTH = 48  # the kernels' path length limit


def start_record() -> np.ndarray:
    rec = np.zeros(66, np.int8)
    back = [4, 2, 3, 5, 6, 3, 2, 4]
    for f in range(8):
        rec[f], rec[8 + f], rec[48 + f], rec[56 + f] = back[f], 1, -1, -back[f]
    rec[64], rec[65] = 15, -1
    return rec


class _Edge:
    __slots__ = ("P", "W", "N", "VL", "child", "action")

    def __init__(self, P, action):
        self.P, self.W, self.N, self.VL, self.child, self.action = P, F(0), 0, 0, None, action


class _Node:
    __slots__ = ("rec", "side", "terminal", "loss", "expanded", "fe", "ne")

    def __init__(self, rec, side, terminal=False, loss=False):
        self.rec, self.side, self.terminal, self.loss = rec, side, terminal, loss
        self.expanded, self.fe, self.ne = False, -1, 0


class _Tree:
    def reset(self, rec, side, move_no):
        self.root = _Node(rec.copy(), int(side))
        self.n = self.vl = 0  # the root's visits and selections in flight
        self.node_count, self.edges, self.move_no = 1, [], move_no
        self.paths = []


class ChessSearch:
    def __init__(self, trees: int, leaves: int = 4, c_puct: float = 1.5, virtual_loss: int = 3,
                 node_capacity: int = 4096):
        self.T, self.L, self.c, self.vlk, self.cap = trees, leaves, F(c_puct), virtual_loss, node_capacity
        self.edge_cap = node_capacity * 64
        self.t = [_Tree() for _ in range(trees)]
        for tr in self.t:
            tr.reset(start_record(), 1, 0)
        self.error = 0

    def set_roots(self, boards: np.ndarray, side: np.ndarray) -> None:
        for tr, b, s in zip(self.t, boards, side):
            tr.reset(np.asarray(b, np.int8), 1 if s >= 0 else -1, 0)

    def _puct(self, e: _Edge, sq):
        vlk = self.vlk * e.VL
        nev = e.N + vlk
        q = (F(e.W) - F(vlk)) / F(nev) if nev > 0 else F(0)
        u1 = self.c * F(e.P)
        u2 = u1 * sq
        u3 = u2 / (F(1) + F(nev))
        return q + u3

    def select(self):
        T, L = self.T, self.L
        boards = np.zeros((T * L, 66), np.int8)
        side = np.zeros(T * L, np.int8)
        term = np.zeros(T * L, np.int8)
        for ti, tr in enumerate(self.t):
            tr.paths = []
            for k in range(L):
                node, np_ = tr.root, tr.n + self.vlk * tr.vl
                tr.vl += 1
                path = []
                while node.expanded and not node.terminal and node.ne > 0:
                    sq = np.sqrt(F(np_))
                    best, bu = -1, None
                    for j in range(node.ne):
                        u = self._puct(tr.edges[node.fe + j], sq)
                        if np.isnan(u):
                            u = F(-np.inf)
                        if bu is None or u > bu:
                            best, bu = j, u
                    e = tr.edges[node.fe + best]
                    if e.child is None and tr.node_count >= self.cap:
                        self.error = self.error or 1
                        break
                    if len(path) + 1 >= MAX_DEPTH:
                        self.error = self.error or 3
                        break
                    c_nv, c_vl = e.N, e.VL
                    e.VL += 1
                    path.append(e)
                    if e.child is None:
                        tr.node_count += 1
                        rec, s = gz.chess_next_state(node.rec, node.side, e.action)
                        oc = gz.chess_ended(rec, s)
                        e.child = _Node(rec, s, terminal=oc != 0, loss=oc == -1)
                    node, np_ = e.child, c_nv + self.vlk * c_vl
                slot = ti * L + k
                boards[slot], side[slot], term[slot] = node.rec, node.side, int(node.terminal)
                legal = (gz.chess_legal_actions(node.rec, node.side) if not node.terminal and not node.expanded
                         else np.zeros(0, np.int16))
                tr.paths.append((path, node, legal))
        return boards, side, term

    def backup(self, pi: np.ndarray, v: np.ndarray) -> None:
        for ti, tr in enumerate(self.t):
            for k, (path, leaf, legal) in enumerate(tr.paths):
                slot = ti * self.L + k
                if leaf.terminal:
                    val = F(-1) if leaf.loss else F(0)
                else:
                    val = F(v[slot])
                    if not leaf.expanded:
                        s = F(0)
                        for a in legal:
                            s = s + F(pi[slot, a])
                        if len(tr.edges) + len(legal) > self.edge_cap:
                            self.error = self.error or 2
                        else:
                            leaf.fe, leaf.ne, leaf.expanded = len(tr.edges), len(legal), True
                            tr.edges += [_Edge(F(pi[slot, a]) / s, int(a)) for a in legal]
                n = len(path)
                for i, e in enumerate(path):
                    x = val if ((n - 1 - i) & 1) else -val
                    e.W = F(e.W) + x
                    e.N += 1
                    e.VL -= 1
                tr.n += 1
                tr.vl -= 1

    def root_edges(self, ti: int) -> list:
        r = self.t[ti].root
        return self.t[ti].edges[r.fe:r.fe + r.ne] if r.expanded else []

    def root_stats(self):
        visits = np.zeros((self.T, gz.CHESS_ACTIONS), np.int32)
        wsum = np.zeros((self.T, gz.CHESS_ACTIONS), np.float32)
        for ti in range(self.T):
            for e in self.root_edges(ti):
                visits[ti, e.action], wsum[ti, e.action] = e.N, e.W
        return visits, wsum

    def tree_sizes(self):
        return (np.array([tr.node_count for tr in self.t], np.int32),
                np.array([len(tr.edges) for tr in self.t], np.int32))

    def choose_greedy(self) -> np.ndarray:
        """The most visited root action, the first in edge order on ties (the
        kernels' rule after the temperature moves)."""
        out = np.zeros(self.T, np.int32)
        for ti in range(self.T):
            es = self.root_edges(ti)
            if es:
                best = 0
                for k, e in enumerate(es):
                    if e.N > es[best].N:
                        best = k
                out[ti] = es[best].action
            else:
                r = self.t[ti].root
                acts = gz.chess_legal_actions(r.rec, r.side)
                out[ti] = int(acts[0]) if len(acts) else 0
        return out

    def play(self, actions: np.ndarray, reserve: int) -> np.ndarray:
        done = np.zeros(self.T, np.int8)
        for ti, tr in enumerate(self.t):
            a, r = int(actions[ti]), tr.root
            ce = next((e for e in self.root_edges(ti) if e.action == a and e.child is not None), None)
            oc = 2
            if a in set(gz.chess_legal_actions(r.rec, r.side).tolist()):
                rec, s = gz.chess_next_state(r.rec, r.side, a)
                oc = gz.chess_ended(rec, s)
            done[ti] = oc != 0
            if oc != 0:
                tr.reset(start_record(), 1, 0)
            elif ce is not None and tr.node_count + reserve <= self.cap:
                tr.root, tr.n, tr.vl, tr.move_no = ce.child, ce.N, ce.VL, tr.move_no + 1
            else:
                tr.reset(rec, s, tr.move_no + 1)
        return done
