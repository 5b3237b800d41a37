"""Contraction trees in omeco's dict format: tc / sc and modeled contraction times.

Same quantities and formats as the reference's ``treesa_gpu.trees`` (treesa_gpu/trees.py:17-149), so that
``optimize`` post-processes its result the same way and callers can compare against it:

* tree dict (omeco ``NestedEinsum.to_dict()``): leaf ``{"tensor_index": i}``, node
  ``{"args": [left, right], "eins": {"ixs": [labels_left, labels_right], "iy": labels_out}}``;
* all indices have dimension 2, so log2 sizes are label counts;
* ``complexity``: tc = log2 sum over contractions of 2^(B+M+N+K), sc = largest tensor (leaves included);
* ``tree_gpu_time`` / ``tree_h100_time``: the reference's two GPU-time models (constants below are the
  reference's model parameters, treesa_gpu/trees.py:87-123).

Every walk here is iterative, so path-like trees with thousands of levels need no recursion limit.
"""
import math

GPU_MODEL = dict(peak_ops=11.9e15, bw_bits=1.6e13, m0=6, n0=6, k0=8, launch=4e-6)
H100_MODEL = dict(launch=4e-6, perm_bw_bits=1.23e13, cc_bit=5.44e-14, cc_cell=7.68e-15, tc_bit=6.37e-14,
                  tc_pad_cell=2.02e-16, tc_out_bit=1.77e-13, small_rank=14, small_cell=1e-12)


def _postorder(d):
    """Nodes of a tree dict in post-order (children before parents), iteratively."""
    out, st = [], [(d, False)]
    while st:
        t, done = st.pop()
        if done or "tensor_index" in t:
            out.append(t)
            continue
        st.append((t, True))
        st.append((t["args"][1], False))
        st.append((t["args"][0], False))
    return out


def leaf_ids(d):
    """Tensor indices of the leaves, left to right."""
    return [t["tensor_index"] for t in _postorder(d) if "tensor_index" in t]


def recompute_outputs(d, ixs, iy):
    """A copy of ``d`` whose internal output labels follow from the topology: a label is an output of a
    node iff it also occurs in a tensor outside the node's subtree, or in the final output ``iy``.
    Labels keep the order of first appearance in (left labels + right labels)."""
    total = {}
    for ix in ixs:
        for l in ix:
            total[l] = total.get(l, 0) + 1
    final = set(iy)
    memo = {}  # id(node) -> (new node, counts, labels)
    for t in _postorder(d):
        if "tensor_index" in t:
            i = t["tensor_index"]
            cnt = {}
            for l in ixs[i]:
                cnt[l] = cnt.get(l, 0) + 1
            memo[id(t)] = ({"tensor_index": i}, cnt, list(ixs[i]))
            continue
        ln, lc, la = memo.pop(id(t["args"][0]))
        rn, rc, lb = memo.pop(id(t["args"][1]))
        if len(lc) < len(rc):
            lc, rc = rc, lc
        for k, v in rc.items():
            lc[k] = lc.get(k, 0) + v
        seen, out = set(), []
        for x in la + lb:
            if x in seen:
                continue
            seen.add(x)
            if x in final or lc[x] < total[x]:
                out.append(x)
        memo[id(t)] = ({"args": [ln, rn], "eins": {"ixs": [la, lb], "iy": out}}, lc, out)
    return memo[id(d)][0]


def contractions(d, ixs):
    """(B, M, N, K) label counts of every pairwise contraction, in post-order."""
    acc, sets = [], {}
    for t in _postorder(d):
        if "tensor_index" in t:
            sets[id(t)] = set(ixs[t["tensor_index"]])
            continue
        a = sets.pop(id(t["args"][0]))
        b = sets.pop(id(t["args"][1]))
        y = set(t["eins"]["iy"])
        acc.append((len(a & b & y), len((a - b) & y), len((b - a) & y), len((a & b) - y)))
        sets[id(t)] = y
    return acc


def complexity(d, ixs):
    """(tc, sc) in log2 units: tc = log2 sum 2^(B+M+N+K), sc = largest tensor, leaves included."""
    cs = contractions(d, ixs)
    if cs:
        mx = max(b + m + n + k for b, m, n, k in cs)
        tc = mx + math.log2(sum(2.0 ** (b + m + n + k - mx) for b, m, n, k in cs))
    else:
        tc = 0.0
    sc = max([b + m + n for b, m, n, k in cs] + [len(set(ix)) for ix in ixs])
    return tc, sc


def gpu_time(B, M, N, K, model=GPU_MODEL):
    """Roofline time model of one contraction (seconds)."""
    ops = 2.0 ** (1 + B + max(M, model["m0"]) + max(N, model["n0"]) + max(K, model["k0"]))
    bits = 2.0 ** (B + M + K) + 2.0 ** (B + N + K) + 2.0 ** (B + M + N)
    return max(ops / model["peak_ops"], bits / model["bw_bits"]) + model["launch"]


def tree_gpu_time(d, ixs, model=GPU_MODEL):
    return sum(gpu_time(*c, model=model) for c in contractions(d, ixs))


def h100_time(B, M, N, K, model=H100_MODEL, small=False):
    """Measured-H100 time model of one contraction (seconds)."""
    if small:
        return model["small_cell"] * 2.0 ** (B + M + N + K)
    a, b, c = 2.0 ** (B + M + K), 2.0 ** (B + N + K), 2.0 ** (B + M + N)
    moved = a + b + c
    perm = 2 * (a + b) / model["perm_bw_bits"]
    best = model["cc_bit"] * moved + model["cc_cell"] * 2.0 ** (B + M + N + K)
    if K >= 7 and max(M, N) >= 5:
        tcv = (model["tc_bit"] * moved + model["tc_pad_cell"] * 2.0 ** (B + max(M, 6) + max(N, 6) + max(K, 8))
               + model["tc_out_bit"] * c)
        best = min(best, tcv)
    return 3 * model["launch"] + perm + best


def tree_h100_time(d, ixs, model=H100_MODEL):
    total = 0.0
    for (B, M, N, K) in contractions(d, ixs):
        total += h100_time(B, M, N, K, model, small=(B + M + N) <= model["small_rank"])
    return total


# names of the reference's modules before its gpu2 -> h100 rename
GPU_MODEL_V2, gpu_time_v2, tree_gpu_time_v2 = H100_MODEL, h100_time, tree_h100_time
