"""Device graph preprocessing (openequivariance_b200.graph) against a scipy construction."""

import numpy as np
import pytest
import torch

from openequivariance_b200.graph import coord_graph, radius_graph


def _scipy_graph(pos, box, cutoff):
    from scipy.spatial import cKDTree

    pairs = cKDTree(pos, boxsize=box).query_pairs(cutoff, output_type="ndarray")
    rows = np.concatenate([pairs[:, 0], pairs[:, 1]])
    cols = np.concatenate([pairs[:, 1], pairs[:, 0]])
    order = np.lexsort((cols, rows))
    rows, cols = rows[order], cols[order]
    return rows, cols, np.lexsort((rows, cols))


@pytest.mark.parametrize("n,box,cutoff", [(400, 12.0, 3.0), (400, 12.0, 5.0), (3000, 20.0, 4.0)])
def test_radius_graph_matches_scipy(n, box, cutoff):
    pos = np.random.default_rng(n).uniform(0, box, size=(n, 3))
    rows, cols, tperm, vec = radius_graph(torch.tensor(pos), box, cutoff)
    r, c, t = _scipy_graph(pos, box, cutoff)
    np.testing.assert_array_equal(rows.numpy(), r)
    np.testing.assert_array_equal(cols.numpy(), c)
    np.testing.assert_array_equal(tperm.numpy(), t)
    d = pos[c] - pos[r]
    d -= box * np.round(d / box)
    np.testing.assert_allclose(vec.numpy(), d, atol=1e-12)


def test_coord_graph_orders():
    rows = torch.tensor([3, 0, 2, 0, 1])
    cols = torch.tensor([1, 2, 0, 1, 3])
    r, c, t, order = coord_graph(rows, cols, 4)
    assert r.tolist() == [0, 0, 1, 2, 3] and c.tolist() == [1, 2, 3, 0, 1]
    assert (rows[order] == r).all() and (cols[order] == c).all()
    key = c[t] * 4 + r[t]
    assert bool((key[1:] > key[:-1]).all())
