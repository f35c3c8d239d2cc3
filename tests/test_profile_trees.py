"""The draft trees of the profiling and benchmark workloads (`profile_decode.tree_of`): n nodes in
breadth-first order, the root with 4 children, each of those with 2, every deeper node with 1, until
there are n nodes; a node's parent comes before it. CPU only."""
from collections import Counter

from seedplane_b200.profile_decode import tree_of
from seedplane_b200.speculative import SpeculativeForest


def _depths(parents):
    d = []
    for p in parents:
        d.append(1 if p < 0 else d[p] + 1)
    return d


def test_tree_shapes():
    for n in (3, 16, 32, 64):
        tokens, parents = tree_of(n, 151936)
        assert len(tokens) == len(parents) == n
        assert all(-1 <= p < i for i, p in enumerate(parents))
        assert all(0 <= t < 151936 for t in tokens)
        kids = Counter(parents)
        assert kids[-1] == min(4, n)
        depths = _depths(parents)
        assert depths == sorted(depths)                      # breadth first
        for i, d in enumerate(depths):
            if d == 1 and kids[i]:
                assert kids[i] <= 2
            if d >= 2:
                assert kids[i] <= 1
    # 32 nodes: 4 + 8 + 8 + 8 + 4 over five levels (the cfg5 tree's depth)
    _, parents = tree_of(32, 1000)
    assert Counter(_depths(parents)) == {1: 4, 2: 8, 3: 8, 4: 8, 5: 4}


def test_tree_paths_rebuild_the_same_forest():
    tokens, parents = tree_of(32, 151936, seed=3)
    chains = []
    for i, p in enumerate(parents):
        chains.append((chains[p] if p >= 0 else ()) + (i,))
    leaves = [i for i in range(32) if i not in set(parents)]
    flat = SpeculativeForest.build([[tokens[j] for j in chains[i]] for i in leaves]).flatten()
    assert sorted(flat.tokens) == sorted(tokens)
    assert sorted(_depths(flat.parents)) == sorted(_depths(parents))
