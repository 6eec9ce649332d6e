"""CPU: the draft-tree topology (breadth-first top-k, truncated) and its
ancestor bit masks; the top-k entry point is exported."""
from cudaforge_b200 import _lib
from cudaforge_b200.tree import topk_tree_shape


def test_444_truncated_to_64():
    sh = topk_tree_shape((4, 4, 4), 64)
    assert sh.nodes == 65
    assert [len(l) for l in sh.levels] == [1, 4, 16, 44]
    assert sh.levels[1] == (1, 2, 3, 4) and sh.levels[2][0] == 5 and sh.levels[3][0] == 21
    for i in range(1, 65):
        assert sh.parent[i] < i and sh.depth[i] == sh.depth[sh.parent[i]] + 1
    # siblings are consecutive in rank order: node 5 + 4j + c is child c of node 1 + j
    for j in range(4):
        for c in range(4):
            assert sh.parent[5 + 4 * j + c] == 1 + j
    # the 44 level-3 nodes hang under the first 11 level-2 nodes
    assert sorted(set(sh.parent[i] for i in sh.levels[3])) == list(range(5, 16))


def test_mask_words_are_ancestor_sets():
    sh = topk_tree_shape((4, 4, 4), 64)
    m = sh.mask_words()
    assert tuple(m.shape) == (65, 2)
    for r in range(65):
        bits = {j for j in range(65) if (int(m[r, j // 64]) >> (j % 64)) & 1}
        anc, j = {r}, r
        while j:
            j = sh.parent[j]
            anc.add(j)
        assert bits == anc, r


def test_branching_one_is_a_chain():
    sh = topk_tree_shape((1, 1, 1, 1), 64)
    assert sh.parent == (0, 0, 1, 2, 3) and sh.depth == (0, 1, 2, 3, 4)


def test_topk_symbol_exported():
    assert hasattr(_lib.lib(), "cf_topk_rows")
