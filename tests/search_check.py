"""Both batch-kernel modes on the same call.

With the visited count or the visited order requested, the search runs the
exact visited set; without them it decides new neighbours by pool membership,
reading each expansion's codes from the copies stored beside the rows (or, with
those freed, gathering them from the code array). `search_both` runs all three
and requires every result they share (ids, distances, counts, ef used,
navigation evaluations, expansions, status) to be identical, then returns the
exact-mode result for the oracle comparison.
"""
import numpy as np

SHARED = ("ids", "dists", "counts", "ef_used", "n_nav", "expansions", "status")


def search_both(dev, q, params, history_cap=0):
    exact = dev.search(q, params, history_cap=history_cap, visited=True)
    fast = dev.search(q, params, visited=False)
    assert "visited" not in fast
    dev.set_fat_rows(False)
    try:
        gathered = dev.search(q, params, visited=False)
    finally:
        dev.set_fat_rows(True)
    for f in SHARED:
        np.testing.assert_array_equal(fast[f], exact[f], err_msg=f"pool-membership mode differs in {f}")
        np.testing.assert_array_equal(gathered[f], exact[f], err_msg=f"gathered-code mode differs in {f}")
    return exact
