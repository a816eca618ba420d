"""Tensor-parallel slicing on CPU (no GPU): which rows and columns of every
tensor each rank keeps (myos_tp_slice, the function myos_load_tensor slices
with), the zero padding of the o_proj input and MLP widths to multiples of
256, and the rank-sliced synthetic generator that feeds a rank only its
block. The reference runs the whole model in one process; the split follows
the heads (q/k/v rows, o_proj columns), the MLP columns (gate/up rows,
down_proj columns) and the untied head's vocabulary rows."""
import os
import socket
import sys

import numpy as np
import pytest

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, os.path.join(REPO, "an-operating-system-for-ai-models-and-tensor-inference_b200"))

from myos import synth  # noqa: E402
from myos.tp import slice_of  # noqa: E402

SPLIT_ROWS = ("q_proj.weight", "q_proj.bias", "k_proj.weight", "k_proj.bias", "v_proj.weight",
              "v_proj.bias", "gate_proj.weight", "up_proj.weight", "lm_head.weight")
SPLIT_COLS = ("o_proj.weight", "down_proj.weight")


def _names(shape, layers=(0,)):
    for name, dims, _ in synth.tensor_specs(shape):
        if name.startswith("model.layers."):
            if int(name.split(".")[2]) not in layers:
                continue
        yield name, dims


def _pad(x):
    return (x + 255) // 256 * 256


@pytest.mark.parametrize("size", [1, 2, 4, 8])
def test_14b_parts_tile_every_tensor_exactly_once(size):
    shape = synth.shape_qwen25_14b()
    for name, dims in _names(shape):
        rows = dims[0]
        cols = dims[1] if len(dims) > 1 else 1
        cover = np.zeros((rows, cols), np.int32) if rows * cols <= 1 << 26 else None
        for rank in range(size):
            p = slice_of(shape, size, rank, name)
            assert p.kept == 1, name
            assert (p.rows, p.cols, p.matrix) == (rows, cols, int(len(dims) > 1)), name
            assert p.row0 + p.nrows <= rows and p.col0 + p.ncols <= cols, name
            assert p.store_rows >= p.nrows and p.store_cols >= p.ncols, name
            split_r = any(name.endswith(s) for s in SPLIT_ROWS)
            split_c = any(name.endswith(s) for s in SPLIT_COLS)
            if size == 1 or not (split_r or split_c):  # whole on every rank
                assert (p.row0, p.nrows, p.col0, p.ncols) == (0, rows, 0, cols), name
                assert (p.store_rows, p.store_cols) == (rows, cols), name
            elif split_r:
                assert (p.nrows, p.row0, p.col0, p.ncols) == (rows // size, rank * (rows // size), 0, cols)
                if name.endswith(("gate_proj.weight", "up_proj.weight")):
                    assert p.store_rows == _pad(rows // size), name  # zero rows pad the MLP width
                else:
                    assert p.store_rows == p.nrows, name
            else:
                assert (p.ncols, p.col0, p.row0, p.nrows) == (cols // size, rank * (cols // size), 0, rows)
                assert p.store_cols == _pad(cols // size), name
            if cover is not None:
                cover[p.row0:p.row0 + p.nrows, p.col0:p.col0 + p.ncols] += 1
        if cover is not None:
            want = size if not any(name.endswith(s) for s in SPLIT_ROWS + SPLIT_COLS) or size == 1 else 1
            assert (cover == want).all(), (name, size)


def test_tied_head_and_unknown_names_are_not_kept():
    shape = synth.shape_qwen25_1_5b()
    for name in ("lm_head.weight", "model.layers.0.self_attn.o_proj.bias", "something.else",
                 "model.layers.99.mlp.up_proj.weight"):
        assert slice_of(shape, 2, 1, name).kept == 0, name


def test_bad_group_is_rejected():
    shape = synth.shape_qwen25_14b()
    with pytest.raises(ValueError):
        slice_of(shape, 3, 0, "model.norm.weight")  # 40 heads do not split 3 ways
    with pytest.raises(ValueError):
        slice_of(shape, 2, 2, "model.norm.weight")


def test_block_generator_matches_the_whole_tensor():
    rows, cols, seed, stream = 37, 101, 1234, 7
    whole = synth.normal_bf16(seed, stream, rows * cols, 0.0, 0.02).reshape(rows, cols)
    for (r0, nr, c0, nc) in [(0, 37, 0, 101), (5, 9, 0, 101), (0, 37, 13, 50), (3, 1, 1, 1),
                             (36, 1, 100, 1)]:
        got = synth.normal_bf16_block(seed, stream, rows, cols, r0, nr, c0, nc, 0.0, 0.02)
        got = got.reshape(rows, cols)
        assert np.array_equal(got[r0:r0 + nr, c0:c0 + nc], whole[r0:r0 + nr, c0:c0 + nc])


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank(rank, world, port, q):
    import datetime

    import torch
    import torch.distributed as dist
    sys.path.insert(0, os.path.join(REPO, "an-operating-system-for-ai-models-and-tensor-inference_b200"))
    from myos import synth as sy
    from myos.tp import slice_of as sl
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60))
    try:
        shape = sy.shape_qwen25_14b()
        out = []
        for name, dims, _ in sy.tensor_specs(shape):
            if not name.startswith(("model.layers.0.", "lm_head", "model.embed")):
                continue
            p = sl(shape, world, rank, name)
            mine = torch.tensor([p.row0, p.nrows, p.col0, p.ncols], dtype=torch.int64)
            parts = [torch.zeros(4, dtype=torch.int64) for _ in range(world)]
            dist.all_gather(parts, mine)
            rows = dims[0]
            cols = dims[1] if len(dims) > 1 else 1
            # every rank sees the same plan: the parts tile the tensor, or all are whole
            area = sum(int(t[1] * t[3]) for t in parts)
            whole = all(int(t[1]) == rows and int(t[3]) == cols for t in parts)
            out.append((name, whole or area == rows * cols))
        q.put((rank, out))
    finally:
        dist.destroy_process_group()


def test_two_gloo_ranks_agree_on_a_tiling():
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=120) for _ in procs)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for rank in (0, 1):
        assert res[rank] and all(ok for _, ok in res[rank]), res[rank]
