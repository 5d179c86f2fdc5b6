"""Speculative-decoding host logic: n-gram draft, exact acceptance, governor hysteresis.

Parity: crates/hawking-speculate/src/user_ngram.rs (propose chain, backoff, smallest-id tie break,
cycle guard), shared.rs:66 (accept until mismatch + correction), governor.rs (streak bail, full
window rate bail, cooldown dwell, enable band).
"""


def test_ngram_chain_backoff_and_tiebreak(native):
    d = native.NgramDraft()
    for t in [1, 2, 3, 4, 1, 2, 3, 5, 1, 2, 3, 4]:
        d.note_token(t)
    # (2,3) -> {4: 2, 5: 1}: 4 wins; (3,4) -> {1}; (4,1) -> {2}
    assert d.propose([2, 3], 4) == [4, 1, 2, 3]
    # unseen bigram context falls back to the unigram successor of the last token
    assert d.propose([9, 3], 1) == [4]
    # nothing recorded after 7: no draft
    assert d.propose([7], 3) == []
    e = native.NgramDraft()
    for t in [1, 8, 1, 6]:  # 1 -> {8: 1, 6: 1}: count tie -> smallest id
        e.note_token(t)
    assert e.propose([1], 1) == [6]


def test_ngram_cycle_guard(native):
    d = native.NgramDraft()
    for _ in range(10):
        d.note_token(7)
    assert d.propose([7, 7], 8) == [7, 7, 7]  # a run of one token stops at 3


def test_accept_draft(native):
    assert native.accept_draft([5, 6, 7], [5, 6, 9, 1]) == ([5, 6, 9], 2)
    assert native.accept_draft([5, 6], [5, 6, 8]) == ([5, 6, 8], 2)  # all accepted + bonus token
    assert native.accept_draft([4], [3, 0]) == ([3], 0)
    assert native.accept_draft([], [11]) == ([11], 0)


def test_governor_hysteresis(native):
    g = native.SpecGovernor(4, 0.25, 3, 2)
    assert g.enabled
    for _ in range(3):
        g.step(False)
    assert not g.enabled  # streak of 3 rejections
    g.step(True)
    assert not g.enabled  # cooldown of 2 recorded cycles
    g.step(True)
    assert g.enabled == (g.accept_rate >= 0.35)
    h = native.SpecGovernor(4, 0.5, 100, 1)
    for a in [True, False, False, True]:
        h.step(a)
    assert not h.enabled  # full window at rate 0.5 <= disable_below
    h.step(True)  # rate 0.5 < 0.6 enable band: stays off after the dwell
    assert not h.enabled
    h.step(True)
    assert h.enabled  # rate 0.75 >= 0.6
