"""Expert-parallel token exchange (test infrastructure: the checker of
b200_ep_dispatch / b200_ep_combine and of the expert-parallel engine).

The reference declares expert parallelism for its MoE layers but never runs
it across devices (atb_cpp_llm/include/atb_llm/layer_desc.h:59-60 names the
expert-parallel fields; atb_cpp_llm/src/components/common/mlp_builder.h:73-82
the MoE MLP); this restates the exchange the B200 path implements, so
"parity" here is an agreed layout, unpinned by reference vectors, checked
through the size-independent property that dispatch -> identity experts ->
combine returns every row times the sum of its routing weights, and that the
expert-parallel MoE equals :func:`oracle.moe.moe_ffn` of the whole model.

Layout: P ranks, E experts, rank d owns experts [d*El, (d+1)*El), El = E/P.
Every source s groups its (token, choice) rows by expert
(:func:`oracle.moe.permute`).  Rank d receives, for each local expert j in
order and, within it, each source rank in order, that source's rows of
expert d*El+j in their grouped order.
"""

import numpy as np

from .moe import permute


def receive_layout(offsets_by_rank, rank):
    """``offsets_by_rank``: every source's ``[E+1]`` group offsets.  Returns
    ``(order, recv_offsets)``: the (source rank, source row) of each received
    row of ``rank`` and the grouped GEMM's ``[El+1]`` group offsets."""
    P = len(offsets_by_rank)
    E = len(offsets_by_rank[0]) - 1
    El = E // P
    order, recv_offsets = [], [0]
    for j in range(El):
        e = rank * El + j
        for s in range(P):
            o = offsets_by_rank[s]
            order += [(s, r) for r in range(int(o[e]), int(o[e + 1]))]
        recv_offsets.append(len(order))
    return order, np.asarray(recv_offsets, np.int32)


def row_base(offsets_by_rank, rank):
    """``[E]``: where ``rank``'s first row of expert e sits in the owner's
    receive buffer (rows of the owner's earlier experts from every source,
    then expert e's rows from lower ranks)."""
    P = len(offsets_by_rank)
    E = len(offsets_by_rank[0]) - 1
    El = E // P
    cnt = np.asarray([np.diff(np.asarray(o, np.int64)) for o in offsets_by_rank])  # [P, E]
    tot = cnt.sum(0)
    out = np.zeros(E, np.int32)
    for e in range(E):
        d0 = (e // El) * El
        out[e] = tot[d0:e].sum() + cnt[:rank, e].sum()
    return out


def dispatch(ids_by_rank, rows_by_rank, num_experts):
    """Every rank's received rows: ``rows_by_rank[s]`` is source s's
    ``[T_s, H]`` tokens, ``ids_by_rank[s]`` its ``[T_s, k]`` expert ids.
    Returns per rank ``(recv [n, H], recv_offsets, row_base)``."""
    P = len(ids_by_rank)
    perms = [permute(ids, num_experts) for ids in ids_by_rank]
    offs = [p[0] for p in perms]
    out = []
    for d in range(P):
        order, ro = receive_layout(offs, d)
        H = rows_by_rank[0].shape[1]
        recv = np.zeros((len(order), H), rows_by_rank[0].dtype)
        for i, (s, r) in enumerate(order):
            recv[i] = rows_by_rank[s][perms[s][2][r]]  # source slot r holds token src[r]
        out.append((recv, ro, row_base(offs, d)))
    return out
