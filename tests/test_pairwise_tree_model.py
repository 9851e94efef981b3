"""The chunk walks of the pairwise order, checked as trees on the CPU.

Dot.pairwise (java/src/main/java/io/drift/kernel/Dot.java:86-102) splits a
count into halves of count >>> 1 down to leaves of at most 8 and combines
left then right. Over a power-of-two depth every split is exact and every
leaf is 8 long, so the kernels walk it in aligned chunks:

- the tiled contraction (gemm.cu) in 16-term tiles: two leaves, one combine,
  then ctz(t + 1) merges of the pending nodes after tile t;
- the one-output-per-thread staged contraction (contract.cu) in 32-term
  chunks: ((leaf0 + leaf1) + (leaf2 + leaf3)), then ctz(c + 1) merges.

Both must build exactly the recursion's tree (the same operands in every
combine, left before right), which these tests compare symbolically."""
import pytest


def recursive_tree(lo, count):
    """Dot.pairwise's tree over terms [lo, lo + count) as nested tuples."""
    if count <= 8:
        return ("leaf", lo, count)
    half = count >> 1
    return (recursive_tree(lo, half), recursive_tree(lo + half, count - half))


def chunk_walk_tree(depth, chunk):
    """The kernels' walk: each aligned chunk's subtree, then ctz(c + 1) merges."""
    def chunk_tree(lo, n):
        if n <= 8:
            return ("leaf", lo, n)
        return (chunk_tree(lo, n // 2), chunk_tree(lo + n // 2, n // 2))

    stack = []
    for c in range(depth // chunk):
        node = chunk_tree(c * chunk, chunk)
        m = c + 1
        while m % 2 == 0:
            node = (stack.pop(), node)
            m //= 2
        stack.append(node)
    assert len(stack) == 1
    return stack[0]


@pytest.mark.parametrize("chunk", [16, 32])
@pytest.mark.parametrize("log_depth", range(4, 15))
def test_chunk_walk_is_the_recursion(chunk, log_depth):
    depth = 1 << log_depth
    if depth < chunk:
        pytest.skip("the walks need at least one whole chunk")
    assert chunk_walk_tree(depth, chunk) == recursive_tree(0, depth)


def _leaves(tree):
    if tree[0] == "leaf":
        return [tree[2]]
    return _leaves(tree[0]) + _leaves(tree[1])


@pytest.mark.parametrize("depth", [48, 96, 100, 1000, 2047, 2049])
def test_other_depths_are_not_chunk_aligned(depth):
    """Why other depths keep the host-built schedule (or the general walk):
    away from powers of two the leaves are shorter than 8 or straddle the
    chunk edges, so chunks are not whole subtrees."""
    counts = _leaves(recursive_tree(0, depth))
    assert sum(counts) == depth
    assert any(c != 8 for c in counts)
