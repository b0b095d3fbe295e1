"""Position math: rope frequency tables, mrope cos/sin, 3-D position ids,
the fp16 causal mask and the 2-D vision rope.

Integer results (``get_rope_index``) are restated exactly; the reference's
tests require a bit-exact match (atb_cpp_llm/tests/level1_cpu_pure/
test_mrope_cpu.cpp:164-166).
"""

import numpy as np


def text_inv_freq(head_dim, theta):
    """inv_freq[i] = 1 / theta^(2i/d), fp32.

    Follows ``TextRotaryEmbedding.__init__``
    (atb_python_qwen3vl_embedding/engine_utils.py:415-427) and
    ``MRoPE::MRoPE`` (atb_cpp_llm/src/components/common/mrope.cpp:16-25).
    """
    e = np.arange(0, head_dim, 2, dtype=np.float32) / np.float32(head_dim)
    return (np.float32(1.0) / np.power(np.float32(theta), e, dtype=np.float32)).astype(np.float32)


def mrope_cos_sin(position_ids, head_dim=128, theta=5e6, sections=(24, 20, 20)):
    """Interleaved 3-section mrope: ``position_ids [3, B, S]`` -> cos, sin ``[B, S, d]``.

    The T plane is the base; index ``i`` (``i % 3 == 1``, ``i < 3*sec[1]``)
    takes the H plane and (``i % 3 == 2``, ``i < 3*sec[2]``) the W plane;
    ``emb = cat(f, f)``.  Restates ``TextRotaryEmbedding.__call__`` /
    ``_apply_interleaved_mrope`` (engine_utils.py:429-457) and
    ``MRoPE::ApplyInterleaved`` / ``MRoPE::Compute`` (mrope.cpp:27-96).
    """
    pid = np.asarray(position_ids, np.int64)
    inv = text_inv_freq(head_dim, theta)
    freqs = pid[..., None].astype(np.float32) * inv  # [3, B, S, d/2]
    f = freqs[0].copy()
    half = head_dim // 2
    for dim, off in ((1, 1), (2, 2)):
        idx = np.arange(off, min(sections[dim] * 3, half), 3)
        f[..., idx] = freqs[dim][..., idx]
    emb = np.concatenate([f, f], -1)
    return np.cos(emb).astype(np.float32), np.sin(emb).astype(np.float32)


def rope1d_cos_sin(positions, head_dim, theta):
    """Standard 1-D rope cos/sin ``[T, d]`` from int positions ``[T]``.

    Restates ``Rope1D::Compute`` (atb_cpp_llm/src/components/common/rope_1d.h:23-167):
    ``freq[t][i] = pos[t] * inv_freq[i]``; ``cos/sin(cat(freq, freq))``.
    """
    inv = text_inv_freq(head_dim, theta)
    f = np.asarray(positions, np.int64)[:, None].astype(np.float32) * inv
    emb = np.concatenate([f, f], -1)
    return np.cos(emb).astype(np.float32), np.sin(emb).astype(np.float32)


def get_rope_index(input_ids, image_grid_thw=None, video_grid_thw=None,
                   attention_mask=None, image_token_id=151655,
                   video_token_id=151656, vision_start_token_id=151652,
                   spatial_merge_size=2):
    """3-D (t, h, w) position ids ``[3, B, S]`` int64 for text + image/video.

    Restates ``get_rope_index`` (atb_python_qwen3vl_embedding/engine_utils.py:469-590)
    and ``GetRopeIndex`` (atb_cpp_llm/src/components/common/mrope.cpp:234-348):
    text runs get sequential ids continuing from the previous chunk's max+1;
    each image/video after a vision-start token gets its merged (t, h, w)
    grid offsets; positions outside the attention mask stay 1.
    """
    ids = np.asarray(input_ids, np.int64)
    B, S = ids.shape
    if video_grid_thw is not None:
        v = np.asarray(video_grid_thw, np.int64)
        v = np.repeat(v, v[:, 0], axis=0)
        v[:, 0] = 1
        video_grid_thw = v
    if image_grid_thw is not None or video_grid_thw is not None:
        img = None if image_grid_thw is None else np.asarray(image_grid_thw, np.int64)
        am = np.ones_like(ids) if attention_mask is None else np.asarray(attention_mask, np.int64)
        pos = np.ones((3, B, S), np.int64)
        image_index = video_index = 0
        for i in range(B):
            toks = ids[i][am[i] == 1].tolist()
            vs = [j for j, t in enumerate(toks) if t == vision_start_token_id]
            vis_tokens = [toks[j + 1] for j in vs if j + 1 < len(toks)]
            if any(j + 1 >= len(toks) for j in vs):
                raise IndexError("vision start token at the end of the sequence")
            image_nums = sum(1 for t in vis_tokens if t == image_token_id)
            video_nums = sum(1 for t in vis_tokens if t == video_token_id)
            chunks = []
            st = 0
            remain_images, remain_videos = image_nums, video_nums
            for _ in range(image_nums + video_nums):
                if image_token_id in toks and remain_images > 0:
                    ed_image = toks.index(image_token_id, st)
                else:
                    ed_image = len(toks) + 1
                if video_token_id in toks and remain_videos > 0:
                    ed_video = toks.index(video_token_id, st)
                else:
                    ed_video = len(toks) + 1
                if ed_image < ed_video:
                    t, h, w = (int(x) for x in img[image_index])
                    image_index += 1
                    remain_images -= 1
                    ed = ed_image
                else:
                    t, h, w = (int(x) for x in video_grid_thw[video_index])
                    video_index += 1
                    remain_videos -= 1
                    ed = ed_video
                gt, gh, gw = t, h // spatial_merge_size, w // spatial_merge_size
                text_len = ed - st
                st_idx = int(chunks[-1].max()) + 1 if chunks else 0
                chunks.append(np.tile(np.arange(text_len, dtype=np.int64), (3, 1)) + st_idx)
                ti = np.repeat(np.arange(gt, dtype=np.int64), gh * gw)
                hi = np.tile(np.repeat(np.arange(gh, dtype=np.int64), gw), gt)
                wi = np.tile(np.arange(gw, dtype=np.int64), gt * gh)
                chunks.append(np.stack([ti, hi, wi]) + text_len + st_idx)
                st = ed + gt * gh * gw
            if st < len(toks):
                st_idx = int(chunks[-1].max()) + 1 if chunks else 0
                chunks.append(np.tile(np.arange(len(toks) - st, dtype=np.int64), (3, 1)) + st_idx)
            llm = np.concatenate(chunks, axis=1).reshape(3, -1)
            pos[:, i, am[i] == 1] = llm
        return pos
    if attention_mask is not None:
        am = np.asarray(attention_mask, np.int64)
        p = np.cumsum(am, -1) - 1
        p[am == 0] = 1
        return np.broadcast_to(p[None], (3, B, S)).copy()
    return np.broadcast_to(np.arange(S, dtype=np.int64)[None, None], (3, B, S)).copy()


def causal_mask_fp16(S):
    """``mask[i][j] = -65504 if j > i else 0`` as fp16 (``MakeCausalMaskFp16``,
    atb_cpp_llm/src/runners/text_runner.cpp:74-85)."""
    m = np.zeros((S, S), np.float16)
    m[np.triu_indices(S, 1)] = np.float16(-65504.0)
    return m


def merge_order(t, h, w, merge_size=2):
    """Row-major patch index (row * w + col) of every token in the vision
    tower's order: merge blocks row-major, the merge_size x merge_size patches
    of a block row-major, the whole grid repeated t times
    (pos_embed_interp.cpp:62-90, engine_utils.py:398-405)."""
    m = merge_size
    order = []
    for br in range(h // m):
        for bc in range(w // m):
            for ir in range(m):
                for ic in range(m):
                    order.append((br * m + ir) * w + bc * m + ic)
    return np.tile(np.asarray(order, np.int64), t)


def pos_embed_interp(table, grid_thw, num_grid=48, merge_size=2):
    """Bilinear interpolation of the learned ``[num_grid^2, H]`` position table
    to each image's ``h x w`` patch grid, in merge order, repeated over t.

    Restates the reference's CPU ``ComputePosEmbedInterp``
    (atb_cpp_llm/src/components/vision/pos_embed_interp.cpp:10-90) in fp32 with
    its exact evaluation order: ``fy = float(i) * (G-1) / (h-1)``, truncating
    floor, ``min(floor+1, G-1)``, and
    ``v00*(1-dy)*(1-dx) + v01*(1-dy)*dx + v10*dy*(1-dx) + v11*dy*dx``.
    The result is fp32 (the reference rounds it to fp16 afterwards).
    """
    table = np.asarray(table, np.float32)
    G = np.float32(num_grid - 1)
    outs = []
    for t, h, w in np.asarray(grid_thw, np.int64):
        def axis(n):
            if n <= 1:
                f = np.zeros(n, np.float32)
            else:
                f = (np.arange(n).astype(np.float32) * G) / np.float32(n - 1)
            lo = f.astype(np.int64)
            hi = np.minimum(lo + 1, num_grid - 1)
            return lo, hi, (f - lo.astype(np.float32)).astype(np.float32)

        y0, y1, dy = axis(int(h))
        x0, x1, dx = axis(int(w))
        one = np.float32(1.0)
        Y0, X0 = np.meshgrid(y0, x0, indexing="ij")
        Y1, X1 = np.meshgrid(y1, x1, indexing="ij")
        DY, DX = np.meshgrid(dy, dx, indexing="ij")
        DY, DX = DY.reshape(-1, 1), DX.reshape(-1, 1)
        v00 = table[(Y0 * num_grid + X0).reshape(-1)]
        v01 = table[(Y0 * num_grid + X1).reshape(-1)]
        v10 = table[(Y1 * num_grid + X0).reshape(-1)]
        v11 = table[(Y1 * num_grid + X1).reshape(-1)]
        interp = (v00 * (one - DY) * (one - DX) + v01 * (one - DY) * DX) + v10 * DY * (one - DX) + v11 * DY * DX
        outs.append(interp[merge_order(int(t), int(h), int(w), merge_size)])
    return np.concatenate(outs).astype(np.float32)


def vision_rope_cos_sin(grid_thw, head_dim=64, merge_size=2, theta=10000.0):
    """2-D vision rope cos/sin ``[T, head_dim]``.

    ``inv_freq = 1/theta^(arange(0, dim, 2)/dim)`` with ``dim = head_dim/2``;
    token order is merge-block major (``(mh, mw, m, m)``), repeated over t;
    ``rope = cat(freq[row], freq[col])``; ``emb = cat(rope, rope)``.
    Restates ``VisionRotaryEmbedding`` / ``compute_rot_pos_emb``
    (engine_utils.py:246-314) and ``ComputeVisionRotPosEmb``
    (atb_cpp_llm/src/components/common/mrope.cpp:155-228).
    """
    dim = head_dim // 2
    e = np.arange(0, dim, 2, dtype=np.float32) / np.float32(dim)
    inv = (np.float32(1.0) / np.power(np.float32(theta), e, dtype=np.float32)).astype(np.float32)
    rows, cols = [], []
    for t, h, w in np.asarray(grid_thw, np.int64):
        mh, mw = h // merge_size, w // merge_size
        r = np.zeros((mh, mw, merge_size, merge_size), np.int64)
        c = np.zeros_like(r)
        for bh in range(mh):
            for bw in range(mw):
                for i in range(merge_size):
                    for j in range(merge_size):
                        r[bh, bw, i, j] = bh * merge_size + i
                        c[bh, bw, i, j] = bw * merge_size + j
        rows.append(np.tile(r.reshape(-1), t))
        cols.append(np.tile(c.reshape(-1), t))
    rows = np.concatenate(rows)
    cols = np.concatenate(cols)
    rope = np.concatenate([rows[:, None].astype(np.float32) * inv,
                           cols[:, None].astype(np.float32) * inv], -1)
    emb = np.concatenate([rope, rope], -1)
    return np.cos(emb).astype(np.float32), np.sin(emb).astype(np.float32)
