"""The speculative-verification oracle on known answers (engine.py:507-520 semantics)."""

from oracle.speculative import accept


def test_accepts_the_longest_matching_prefix():
    # Row 0: drafts [7, 8, 9] after pending 5; predictions after 5, 7, 8, 9 are [7, 8, 4, 1]:
    # drafts 7 and 8 match, 9 != 4 -> accepted 2, emits [7, 8, 4].
    # Row 1: one logit row (a plain decode or prefill row) -> emits its head.
    # Row 2: first draft already differs -> accepted 0, emits the first prediction only.
    chunks = [[5, 7, 8, 9], [11], [3, 6, 6]]
    logit_counts = [4, 1, 3]
    predictions = [7, 8, 4, 1, 42, 2, 6, 6]
    accepted, emitted = accept(chunks, logit_counts, predictions)
    assert accepted == [2, 0, 0]
    assert emitted == [[7, 8, 4], [42], [2]]


def test_full_acceptance_emits_the_bonus_token():
    accepted, emitted = accept([[1, 2, 3]], [3], [2, 3, 9])
    assert accepted == [2] and emitted == [[2, 3, 9]]
