"""Both batch-kernel modes on the same call.

With the visited count or the visited order requested, the search runs the
exact visited set; without them it decides new neighbours by pool membership.
`search_both` runs both and requires every result they share (ids,
distances, counts, ef used, navigation evaluations, expansions, status) to be
identical, then returns the exact-mode result for the oracle comparison.
"""
import numpy as np

SHARED = ("ids", "dists", "counts", "ef_used", "n_nav", "expansions", "status")


def search_both(dev, q, params, history_cap=0):
    exact = dev.search(q, params, history_cap=history_cap, visited=True)
    fast = dev.search(q, params, visited=False)
    assert "visited" not in fast
    for f in SHARED:
        np.testing.assert_array_equal(fast[f], exact[f], err_msg=f"pool-membership mode differs in {f}")
    return exact
