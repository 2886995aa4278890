"""Known-answer checks of the CPU showdown restatement (no GPU).

The external evaluator is not available, so its ranking is restated: these
cases pin the standard order on the full deck and the rarity order of
pbg's cards.py:37-74 on short decks.
"""

import numpy as np

import oracle as O


def card(rank: str, suit: int) -> int:
    return 4 * "23456789TJQKA".index(rank) + suit


def value(R, cards):
    return O.hand_value7(R, [card(r, s) for r, s in cards])


def test_full_deck_category_order():
    R = 13
    royal = value(R, [("A", 0), ("K", 0), ("Q", 0), ("J", 0), ("T", 0), ("2", 1), ("3", 2)])
    quads = value(R, [("A", 0), ("A", 1), ("A", 2), ("A", 3), ("K", 0), ("2", 1), ("3", 2)])
    boat = value(R, [("A", 0), ("A", 1), ("A", 2), ("K", 3), ("K", 0), ("2", 1), ("3", 2)])
    flush = value(R, [("A", 0), ("9", 0), ("7", 0), ("5", 0), ("3", 0), ("2", 1), ("K", 2)])
    wheel = value(R, [("A", 0), ("2", 1), ("3", 2), ("4", 3), ("5", 0), ("9", 1), ("J", 2)])
    six_high = value(R, [("6", 0), ("2", 1), ("3", 2), ("4", 3), ("5", 0), ("9", 1), ("J", 2)])
    trips = value(R, [("7", 0), ("7", 1), ("7", 2), ("A", 3), ("K", 0), ("2", 1), ("4", 2)])
    assert royal > quads > boat > flush > six_high > wheel > trips


def test_short_deck_flush_beats_full_house_when_rarer():
    # R=8 (ranks 6..A): flush (224 combos) is rarer than a full house (1344)
    R = 8
    flush = value(R, [("A", 0), ("Q", 0), ("T", 0), ("8", 0), ("6", 0), ("K", 1), ("K", 2)])
    boat = value(R, [("K", 0), ("K", 1), ("K", 2), ("Q", 3), ("Q", 1), ("6", 1), ("7", 2)])
    assert flush > boat
    # R=13: the usual order
    assert value(13, [("A", 0), ("Q", 0), ("T", 0), ("8", 0), ("6", 0), ("K", 1), ("K", 2)]) < value(
        13, [("K", 0), ("K", 1), ("K", 2), ("Q", 3), ("Q", 1), ("6", 1), ("7", 2)])


def test_no_wheel_on_short_decks():
    # with R=9 the deck is 6..A; A-6-7-8-9 is not a straight
    R = 9
    v = value(R, [("A", 0), ("6", 1), ("7", 2), ("8", 3), ("9", 0), ("J", 1), ("Q", 2)])
    s = value(R, [("T", 0), ("6", 1), ("7", 2), ("8", 3), ("9", 0), ("J", 1), ("2", 2)])
    assert s > v


def test_split_pot_shares_equally():
    R = 13
    geom = O.Geometry(3, 8.0, R)
    m = O.Machine(geom)
    board = np.array([[card("A", 0), card("K", 1), card("Q", 2), card("J", 3), card("T", 0)]], np.uint8)
    combo = m.combo_id(np.array([card("2", 0), card("2", 1), card("3", 0)]),
                       np.array([card("3", 1), card("4", 1), card("4", 2)]))[None]
    level = np.zeros((1, 3), np.int32)
    base = -np.full((1, 3), 4.0, np.float32)
    amount = np.array([[12.0, 0.0, 0.0]], np.float32)
    pay = O.evaluate_showdowns(R, board, combo, level, base, amount)
    np.testing.assert_allclose(pay, [[0.0, 0.0, 0.0]])
    level[0, 2] = -1
    pay = O.evaluate_showdowns(R, board, combo, level, base, amount)
    np.testing.assert_allclose(pay, [[2.0, 2.0, -4.0]])
