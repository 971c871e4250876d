"""Tensor-parallel layers, collectives and topology (CPU; gloo multi-process where needed)."""
import torch
import torch.distributed as dist

from dist_util import run_ranks
from mini_megatron_b200.comm.mappings import (AllReduce, all_reduce, copy_to_model_parallel_region,
                                              reduce_from_model_parallel_region)
from mini_megatron_b200.parallel.process_groups import rank_coords
from mini_megatron_b200.parallel.tensor_parallel import (ColumnParallelLinear, RowParallelLinear,
                                                         VocabParallelEmbedding, pad_vocab_size,
                                                         strided_gather_rows, strided_partition_rows)


def test_column_parallel_equals_linear_at_tp1():
    torch.manual_seed(0)
    full = torch.nn.Linear(64, 32, bias=False)
    col = ColumnParallelLinear(64, 32, bias=False)
    with torch.no_grad():
        col.weight.copy_(full.weight)
    x = torch.randn(2, 8, 64)
    torch.testing.assert_close(col(x), full(x))


def test_row_parallel_equals_linear_at_tp1():
    torch.manual_seed(0)
    full = torch.nn.Linear(64, 32, bias=False)
    row = RowParallelLinear(64, 32, bias=False)
    with torch.no_grad():
        row.weight.copy_(full.weight)
    x = torch.randn(2, 8, 64)
    torch.testing.assert_close(row(x), full(x))


def test_qkv_strided_partition_keeps_q_k_v_on_every_rank():
    rows = torch.arange(12).reshape(12, 1)
    assert strided_partition_rows(rows, 2, 0, stride=3).flatten().tolist() == [0, 1, 4, 5, 8, 9]
    assert strided_partition_rows(rows, 2, 1, stride=3).flatten().tolist() == [2, 3, 6, 7, 10, 11]
    shards = [strided_partition_rows(rows, 2, r, stride=3) for r in range(2)]
    assert torch.equal(strided_gather_rows(shards, stride=3), rows)


def test_vocab_parallel_embedding_matches_embedding_at_tp1():
    torch.manual_seed(7)
    full = torch.nn.Embedding(16, 4)
    par = VocabParallelEmbedding(16, 4)
    with torch.no_grad():
        par.weight.copy_(full.weight)
    tokens = torch.tensor([[0, 3, 9, 15]])
    assert torch.equal(par(tokens), full(tokens))


def test_pad_vocab_size():
    assert pad_vocab_size(50257, 1) == 50304
    assert pad_vocab_size(50257, 8) == 51200
    assert pad_vocab_size(1024, 2) == 1024


def test_all_reduce_passthrough_when_no_group():
    x = torch.randn(4)
    torch.testing.assert_close(all_reduce(x, None), x)
    assert AllReduce is not None


def test_rank_coords_match_reference_layout():
    # rank = dp*(tp*pp) + pp*tp + tp
    tp, pp = 2, 2
    coords = [rank_coords(r, tp, pp) for r in range(8)]
    assert coords[0] == (0, 0, 0) and coords[1] == (1, 0, 0) and coords[2] == (0, 1, 0)
    assert coords[5] == (1, 0, 1) and coords[7] == (1, 1, 1)


def _topology_worker(rank, world, tp, pp):
    from mini_megatron_b200.parallel.process_groups import init_model_parallel
    mpu = init_model_parallel(tp, pp)
    return {k: mpu[k] for k in ("tp_rank", "pp_rank", "dp_rank", "tp_ranks", "pp_ranks", "dp_ranks")}


def test_topology_groups_tp2_pp2_dp2():
    res = run_ranks(_topology_worker, 8, 2, 2)
    assert res[0]["tp_ranks"] == [0, 1] and res[0]["pp_ranks"] == [0, 2] and res[0]["dp_ranks"] == [0, 4]
    assert res[5]["tp_ranks"] == [4, 5] and res[5]["pp_ranks"] == [5, 7] and res[5]["dp_ranks"] == [1, 5]
    for r, d in enumerate(res):
        assert r in d["tp_ranks"] and r in d["pp_ranks"] and r in d["dp_ranks"]


def _tp_linear_worker(rank, world):
    # Column (2 rows per rank) followed by Row (2 input columns per rank).
    x = torch.tensor([[1.0, -2.0, 3.0, 0.5]], requires_grad=True)
    w_col = torch.arange(16.0).reshape(4, 4) / 10
    w_row = torch.arange(16.0).reshape(4, 4) / 7
    cs = w_col[rank * 2:(rank + 1) * 2].clone().requires_grad_(True)
    rs = w_row[:, rank * 2:(rank + 1) * 2].clone().requires_grad_(True)
    h = torch.nn.functional.linear(copy_to_model_parallel_region(x, dist.group.WORLD), cs)
    out = reduce_from_model_parallel_region(torch.nn.functional.linear(h, rs), dist.group.WORLD)
    out.sum().backward()
    return {"x_grad": x.grad, "col": cs.grad, "row": rs.grad}


def test_tp_autograd_matches_full_two_linear_reference():
    x = torch.tensor([[1.0, -2.0, 3.0, 0.5]], requires_grad=True)
    wc = (torch.arange(16.0).reshape(4, 4) / 10).requires_grad_(True)
    wr = (torch.arange(16.0).reshape(4, 4) / 7).requires_grad_(True)
    torch.nn.functional.linear(torch.nn.functional.linear(x, wc), wr).sum().backward()
    states = run_ranks(_tp_linear_worker, 2)
    for r, s in enumerate(states):
        torch.testing.assert_close(s["x_grad"], x.grad)
        torch.testing.assert_close(s["col"], wc.grad[r * 2:(r + 1) * 2])
        torch.testing.assert_close(s["row"], wr.grad[:, r * 2:(r + 1) * 2])


def test_compute_mfu_dp_cancels_and_caps():
    from mini_megatron_b200.config import get_model_config
    from mini_megatron_b200.training import compute_mfu
    c = get_model_config()
    a = compute_mfu(c, 512, 4, 1, 1, 1.0, 100)
    b = compute_mfu(c, 512, 4, 1, 1, 0.5, 50)
    assert abs(a - b) < 1e-9
    assert compute_mfu(c, 512, 4, 1, 1, 1e-6, 100) <= 1.0
