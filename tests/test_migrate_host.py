"""Host side of the hot -> cold migration cycle: candidate choice
(distiller.rs:115-121) and the page-table rewrite.  CPU only."""
import numpy as np

from aether_nexus_b200 import migrate


def test_choose_candidates_window_and_flags():
    ent = np.array([0.0, 0.1, 0.2, 0.05, 0.149, 0.15, 0.01], np.float32)
    hot_refs = np.array([0, 1, 2, 3 | (1 << 31), 4, 5, 6], np.uint32)
    hot_indptr = np.array([0, 4, 7], np.uint32)
    got = migrate.choose_candidates(ent, hot_refs, hot_indptr, 0.15, keep_recent=1)
    # seq 0: positions 0..2 considered (3 is the newest), block 0 has proxy 0,
    # block 2 is above the threshold -> only position 1
    # seq 1: positions 4..5 considered, 0.149 < 0.15 but 0.15 is not
    assert got == [[1], [4]]
    assert migrate.choose_candidates(ent, hot_refs, hot_indptr, 0.15, keep_recent=0) == [[1, 3], [4, 6]]
    # a reference outside the proxy array is never a candidate
    assert migrate.choose_candidates(ent[:2], hot_refs, hot_indptr, 0.15, keep_recent=0) == [[1], []]


def test_rewrite_page_tables_conserves_blocks():
    hot_refs = np.array([10, 11, 12, 20, 21], np.uint32)
    hot_indptr = np.array([0, 3, 5], np.uint32)
    cold_refs = np.array([1, 2, 3], np.uint32)
    cold_indptr = np.array([0, 2, 3], np.uint32)
    nh, hip, nc, cip = migrate.rewrite_page_tables(hot_refs, hot_indptr, cold_refs, cold_indptr, [[0, 2], [3]],
                                                   [7, 8, 9])
    assert nh.tolist() == [11, 21] and hip.tolist() == [0, 1, 2]
    assert nc.tolist() == [1, 2, 7, 8, 3, 9] and cip.tolist() == [0, 4, 6]
    # nothing moved: tables unchanged
    nh, hip, nc, cip = migrate.rewrite_page_tables(hot_refs, hot_indptr, cold_refs, cold_indptr, [[], []], [])
    assert nh.tolist() == hot_refs.tolist() and nc.tolist() == cold_refs.tolist()
    assert hip.tolist() == hot_indptr.tolist() and cip.tolist() == cold_indptr.tolist()
