"""Known-answer rule scenarios as TorchEnv50 rows (test infrastructure).

The reference pins its rarer rules with hand-built states (tests/hangame_rules50_test.cpp,
special50_test.cpp, terminal50_test.cpp): a neutral ppuk captured, the last turns'
ppuk and steal rules, a hand bonus on the last turn, a first-turn ttadak, a third
ppuk, a bonus replacement that completes a month in hand, forced bombs and
four-card shakes.  Those tests drive the reference's inner state layers; here each
case is restated as a decision point of the row the engines step -- the cards placed
as the case needs, every other card in the stock, and the stock's random stream
chosen so that the flip shows the case's card -- so the same situation is stepped by
the reference engine (the oracle), the host build of this engine's headers and the
GPU kernels.
"""
from __future__ import annotations

from dataclasses import dataclass, field

import numpy as np

DECK = (1 << 50) - 1
DONE_BYTE = 239  # TorchEnv50::done
WORDS = 31


def card(month: int, slot: int) -> int:
    return 4 * month + slot


def bits(*cards: int) -> int:
    m = 0
    for c in cards:
        m |= 1 << c
    return m


def pi_cards(first_month: int, count: int) -> list[int]:
    """Plain pi (slots 2 and 3) from `first_month` on, as the reference's helper."""
    out, month = [], first_month
    while count > 0:
        for slot in (2, 3):
            if count > 0:
                out.append(card(month, slot))
                count -= 1
        month += 1
    return out


def _put(w: np.ndarray, word: int, shift: int, width: int, value: int) -> None:
    mask = ((1 << width) - 1) << shift
    w[word] = np.uint64((int(w[word]) & ~mask & (2**64 - 1)) | ((int(value) << shift) & mask))


def _get(w: np.ndarray, word: int, shift: int, width: int) -> int:
    return (int(w[word]) >> shift) & ((1 << width) - 1)


@dataclass
class Case:
    """One scenario: where the cards lie, the flags that differ from a fresh turn, the
    card the stock flip must show, and the actions to take in order."""
    name: str
    hand0: list[int]
    hand1: list[int]
    floor: list[int]
    actions: list[int]
    pile0: list[int] = field(default_factory=list)
    pile1: list[int] = field(default_factory=list)
    turn: int = 0
    neutral_ppuk: int = 0       # month bits
    ppuk_streak0: int = 0
    credits0: int = 0
    flip: int | None = None     # the first stock draw


def fresh_row(oracle) -> np.ndarray:
    """A dealt, running game with player 0 to move (the base every case edits)."""
    seeds = np.arange(12345, 12345 + 64, dtype=np.int64)
    rows = oracle.create(seeds, np.zeros(64, dtype=np.int64))
    w = rows.view(np.uint64).reshape(64, WORDS)
    for i in range(64):
        if rows[i, 239] == 0 and _get(w[i], 16, 8, 8) == 0 and _get(w[i], 27, 24, 8) == 0:
            return rows[i].copy()
    raise RuntimeError("no running deal among the first 64 seeds")


def build(case: Case, base: np.ndarray, engine) -> np.ndarray:
    """The case as a row: cards placed, every unplaced card in the stock, missions and
    prompts cleared, player 0 at a primary decision on turn `case.turn`; the stock's
    random stream is the first whose next draw is `case.flip` (found with the
    engine's stock preview)."""
    row = base.copy()
    w = row.view(np.uint64)
    placed = {k: bits(*getattr(case, k)) for k in ("hand0", "hand1", "floor", "pile0", "pile1")}
    total = 0
    for m in placed.values():
        assert total & m == 0, f"{case.name}: a card placed twice"
        total |= m
    stock = DECK & ~total
    w[0], w[1], w[2], w[3] = placed["hand0"], placed["hand1"], placed["floor"], stock
    w[4], w[5] = placed["pile0"], placed["pile1"]
    w[7] = 0                                    # flip bonus
    w[8] = 0                                    # ppuk months, owner/Gukjin flags, ppuk bonus
    _put(w, 9, 0, 16, case.turn)
    _put(w, 9, 16, 8, 0)                        # actor 0
    _put(w, 9, 24, 8, 0)                        # play phase
    _put(w, 9, 32, 8, 0xFF)                     # no played card
    _put(w, 9, 40, 8, 0xFF)                     # no drawn card
    w[10] = 0                                   # no mission cards
    _put(w, 11, 0, 16, case.neutral_ppuk)
    _put(w, 12, 0, 32, 0)                       # Go counts and last Go scores
    _put(w, 12, 32, 8, 0xFF)                    # no Go/Stop prompt
    _put(w, 12, 40, 8, 0xFF)                    # no winner
    _put(w, 12, 48, 8, 0)                       # no Gukjin prompt
    w[13] = 0                                   # shakes, bombs, credits
    _put(w, 13, 48, 8, case.credits0)
    w[14] = 0                                   # four-card shakes
    _put(w, 15, 0, 32, case.ppuk_streak0 << 16)  # ppuk counts 0, streaks
    _put(w, 15, 32, 8, 0xFF)                    # no Chongtong prompt
    _put(w, 15, 48, 16, 0)
    _put(w, 16, 0, 8, 0xFF)                     # no end
    _put(w, 16, 8, 8, 0)
    w[17] = 0
    _put(w, 18, 0, 32, 0)                       # side payments
    _put(w, 18, 40, 24, 0)                      # mission type, multipliers
    _put(w, 19, 0, 8, 0)
    w[20], w[21] = placed["hand0"], placed["hand1"]  # cards ever held
    w[22], w[23] = 0, 0                         # cards shown
    if case.flip is not None:
        cands = np.repeat(row[None, :], 4096, axis=0)
        cw = cands.view(np.uint64).reshape(4096, WORDS)
        cw[:, 6] = np.arange(1, 4097, dtype=np.uint64) * np.uint64(0x9E3779B97F4A7C15)
        first = engine.stock(cands) & 0xFF
        hit = np.flatnonzero(first == case.flip)
        assert hit.size, f"{case.name}: no stream flips card {case.flip}"
        w[6] = cw[hit[0], 6]
    return row


# Filler cards: months 10 and 11 stay out of every case's play.
_F0 = [card(10, 0), card(10, 1)]
_F1 = [card(11, 0), card(11, 1), card(10, 2)]

CASES = [
    # hangame_rules50_test.cpp:93-109 -- capturing a dealt triple steals one pi.
    Case("neutral_ppuk_capture", hand0=[card(3, 3)] + _F0, hand1=_F1,
         floor=[card(3, 0), card(3, 1), card(3, 2), card(9, 0)], pile1=pi_cards(6, 2),
         neutral_ppuk=1 << 3, flip=card(5, 0), actions=[card(3, 3)]),
    # :125-133 -- a jjok on the last turn takes the cards but steals nothing.
    Case("last_turn_jjok", hand0=[card(0, 0)], hand1=[card(11, 0)], floor=[card(1, 0)],
         pile1=pi_cards(6, 2), turn=18, flip=card(0, 1), actions=[card(0, 0)]),
    # :135-143 -- a would-be ppuk on the last turn is captured instead.
    Case("last_turn_ppuk", hand0=[card(1, 1)], hand1=[card(11, 0)], floor=[card(1, 0)],
         pile1=pi_cards(6, 2), turn=18, flip=card(1, 2), actions=[card(1, 1)]),
    # :145-150 -- the same play before the last turns makes a ppuk.
    Case("ppuk_before_last_turn", hand0=[card(1, 1)] + _F0, hand1=_F1, floor=[card(1, 0)],
         pile1=pi_cards(6, 2), turn=16, flip=card(1, 2), actions=[card(1, 1)]),
    # :152-162 -- a hand bonus on the last turn steals nothing.
    Case("last_turn_bonus", hand0=[48, card(10, 0)], hand1=[card(11, 0)], floor=[card(9, 0)],
         pile1=[card(1, 2)], turn=18, flip=card(0, 0), actions=[48]),
    # :385-433 -- a first-turn ttadak captures four cards, steals and pays 7.
    Case("first_turn_ttadak", hand0=[card(2, 2)] + _F0, hand1=_F1,
         floor=[card(2, 0), card(2, 1), card(9, 0)], pile1=pi_cards(6, 2), turn=0,
         flip=card(2, 3), actions=[card(2, 2)]),
    # terminal50_test.cpp:154-211 -- the third ppuk of an opening streak ends the game.
    Case("third_ppuk", hand0=[card(1, 1)] + _F0, hand1=_F1, floor=[card(1, 0)], turn=4,
         ppuk_streak0=2, flip=card(1, 2), actions=[card(1, 1)]),
    # terminal50_test.cpp:119-152 -- a bonus replacement completing a month in hand
    # offers a Chongtong; taking it ends the game.
    Case("bonus_replacement_chongtong", hand0=[48, card(0, 0), card(0, 1), card(0, 2)],
         hand1=_F1, floor=[card(9, 0)], flip=card(0, 3), actions=[48, 125]),
    # hangame_rules50_test.cpp:293-336 -- three in hand and one on the floor: the bomb
    # is forced (single plays of the month are not legal), then played.
    Case("forced_bomb", hand0=[card(4, 0), card(4, 1), card(4, 2)] + _F0, hand1=_F1,
         floor=[card(4, 3), card(9, 0)], pile1=pi_cards(6, 2), flip=card(5, 0),
         actions=[card(4, 0), 98 + 4]),
    # :293-336 -- a whole month in hand with none on the floor offers a four-card shake.
    Case("four_card_shake", hand0=[card(4, 0), card(4, 1), card(4, 2), card(4, 3)] + _F0,
         hand1=_F1, floor=[card(9, 0)], flip=card(5, 0), actions=[50 + card(4, 0)]),
    # A bomb credit: one card flipped and resolved, the credit spent.
    Case("bomb_credit", hand0=_F0, hand1=_F1, floor=[card(9, 0)], credits0=1,
         flip=card(9, 1), actions=[122]),
]


def play(case_rows: np.ndarray, actions: list[int], step) -> list[tuple]:
    """Steps the rows through `step(rows, actions)` once per action; the outputs."""
    out, rows = [], case_rows
    for a in actions:
        res = step(rows, np.full(rows.shape[0], a, dtype=np.int64))
        out.append(res)
        rows = res[0]
    return out
