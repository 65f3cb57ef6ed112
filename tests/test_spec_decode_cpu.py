"""Host logic of the self-speculative decode harness (no GPU): the per-step
shapes of the fixed-draft schedule and the acceptance rule."""

import numpy as np

from aspire_b200.spec_decode import accept, compare_sequences, step_shape


def test_accept_is_the_longest_matching_prefix():
    assert accept(np.array([5, 6, 7, 8]), np.array([5, 6, 9, 8, 1])) == 2
    assert accept(np.array([5, 6, 7, 8]), np.array([5, 6, 7, 8, 1])) == 4
    assert accept(np.array([5]), np.array([4, 1])) == 0
    assert accept(np.array([], np.int64), np.array([3])) == 0


def test_step_shape_draft_verify_and_finished_rows():
    D, k = 4, 8
    n = np.array([100, 100, 31, 500, 40])
    dcnt = np.array([0, 4, 2, 4, 1])
    active = np.array([True, True, True, True, False])
    s = step_shape(n, dcnt, active, D, k)
    # row 0 drafts at position 100; row 1 verifies 5 tokens at 100..104
    assert s["draft"].tolist() == [True, False, True, False, False]
    assert s["verify"].tolist() == [False, True, False, True, False]
    assert s["qlen"].tolist() == [1, 5, 1, 5, 0]
    assert s["start"].tolist() == [100, 100, 33, 500, 40]
    assert s["end"].tolist() == [101, 105, 34, 505, 40]
    assert s["qo"].tolist() == [0, 1, 6, 7, 12, 12]
    # draft rows: min(ceil(end / 16), k) pages ending with the page of end - 1
    assert s["mixed_pages"].tolist() == [7, 7, 3, 32, 3]
    assert s["last"].tolist() == [5, 9, 2, 9, 8]
    assert s["mixed_len"].tolist() == [6 * 16 + 5, 105, 2 * 16 + 2, 505, 40]
    # a budget smaller than the pages: the draft row sees budget pages
    s2 = step_shape(np.array([1000]), np.array([0]), np.array([True]), D, 8)
    assert s2["mixed_pages"].tolist() == [8] and s2["mixed_len"].tolist() == [7 * 16 + (1000 % 16) + 1]


def test_compare_sequences():
    a = np.array([[1, 2, 3], [1, 2, 3]])
    b = np.array([[1, 2, 3], [1, 5, 3]])
    r = compare_sequences(a, b)
    assert r["rows_identical"] == 1 and r["first_divergence"] == [-1, 1]
