"""CPU: tensor-parallel sharding of RVQ entries is exact, and a 2-rank
column-/row-parallel layer (gloo all-reduce) equals the unsharded layer."""

import os

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from oracle.rvq_oracle import OUT_F32, RVQEntryNP, decode_rvq
from rvq_b200 import shard, synthetic


def recon(entry, cb):
    rows, cols = entry["shape"]
    e = RVQEntryNP(indices=entry["indices"].numpy(), codebook=cb.float().numpy(),
                   scales=entry["scales"].float().numpy(), tail=entry["tail"].float().numpy(), d=8,
                   group_size=int(entry["group_size"]), trimmed_numel=int(entry["trimmed_numel"]),
                   numel=rows * cols)
    return decode_rvq(e, OUT_F32).reshape(rows, cols)


@pytest.mark.parametrize("rows,cols,group,tp", [(512, 256, None, 2), (512, 256, 64, 4), (96, 1024, 128, 8),
                                                (64, 512, 1024, 2)])
def test_row_and_column_shards_are_exact_slices(rows, cols, group, tp):
    g = torch.Generator().manual_seed(rows + cols + tp)
    cb = synthetic.make_codebook(4, 256, 8, g)
    e = synthetic.make_rvq_entry(rows, cols, g, group_size=group)
    full = recon(e, cb)
    for r in range(tp):
        rs = shard.shard_rows(e, r, tp)
        assert np.array_equal(recon(rs, cb), full[r * rows // tp:(r + 1) * rows // tp])
        cs = shard.shard_cols(e, r, tp)
        assert np.array_equal(recon(cs, cb), full[:, r * cols // tp:(r + 1) * cols // tp])


def test_straddling_scale_groups_are_refused():
    g = torch.Generator().manual_seed(1)
    e = synthetic.make_rvq_entry(6, 256, g, group_size=256 * 3)        # 3 rows per scale
    with pytest.raises(ValueError):
        shard.shard_rows(e, 0, 3)                                      # 2-row shards cut a scale
    e2 = synthetic.make_rvq_entry(64, 384, g, group_size=128)
    with pytest.raises(ValueError):
        shard.shard_cols(e2, 0, 2)                                     # 192-column shards cut a group
    with pytest.raises(ValueError):
        shard.sharded_dims(32, 8, 9728, 16)


def _layer_worker(rank, world, port, out):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    g = torch.Generator().manual_seed(0)
    shape = synthetic.BlockShape(hidden=256, intermediate=512, n_heads=4, n_kv_heads=2, head_dim=64)
    cbs = synthetic.make_family_codebooks(g)
    entries = synthetic.make_block_entries(shape, 0, g)
    mine = shard.shard_layer(entries, 0, rank, world)
    x = torch.randn(256, generator=torch.Generator().manual_seed(5), dtype=torch.float64)
    W = lambda ents, n: torch.from_numpy(recon(ents[f"model.layers.0.{n}"],
                                               cbs[synthetic.FAMILY_OF[n]])).double()
    # column-parallel gate/up, local SiLU product, row-parallel down + all-reduce
    gate = W(mine, "mlp.gate_proj.weight") @ x
    up = W(mine, "mlp.up_proj.weight") @ x
    act = torch.nn.functional.silu(gate) * up
    y = W(mine, "mlp.down_proj.weight") @ act
    dist.all_reduce(y)
    full_act = torch.nn.functional.silu(W(entries, "mlp.gate_proj.weight") @ x) * (W(entries, "mlp.up_proj.weight") @ x)
    want = W(entries, "mlp.down_proj.weight") @ full_act
    out[rank] = float((y - want).abs().max() / want.abs().max())
    dist.destroy_process_group()


def test_two_rank_mlp_equals_unsharded():
    ctx = mp.get_context("spawn")
    out = ctx.Manager().dict()
    port = 29500 + os.getpid() % 1000
    procs = [ctx.Process(target=_layer_worker, args=(r, 2, port, out)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    assert max(out.values()) < 1e-12
