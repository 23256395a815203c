"""Fused weight broadcast: the job planner on CPU (restated in PyTorch), the
kernel on one GPU against the PyTorch conversion, and the multicast / peer
broadcast on two GPUs (child processes)."""
import os
import subprocess
import sys

import pytest
import torch

from connex_b200.models.llama import LlamaConfig, LlamaWeights, random_trainer_weights, trainer_layout
from connex_b200.parallel.wsync import emulate_jobs, engine_manifest, fuse_reference, plan_jobs

CFG = LlamaConfig.tiny(layers=2)


def _engine_bytes(cfg, fused, manifest):
    out = torch.zeros(manifest.total, dtype=torch.uint8)
    for e in manifest.entries:
        out[e.offset:e.offset + e.nbytes] = fused[e.name].detach().cpu().contiguous().view(-1).view(torch.uint8)
    return out


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_plan_matches_pytorch_fusion(dtype):
    named = random_trainer_weights(CFG, "cpu", dtype=dtype)
    m = engine_manifest(CFG)
    jobs, n_tasks, srcs = plan_jobs(CFG, m, named, task_bytes=4096)
    assert jobs[:, 10].tolist() == sorted(jobs[:, 10].tolist()) and n_tasks > len(named)
    got = emulate_jobs(jobs, srcs, m.total)
    want = _engine_bytes(CFG, fuse_reference(CFG, named), m)
    assert torch.equal(got, want)
    w = LlamaWeights.from_arena(CFG, got, m)
    assert w.layers[1].w13.shape == (2 * CFG.ffn, CFG.hidden)


def test_relay_plan_covers_the_arena_once():
    """The relay's forward intervals, over all rounds and slice owners, are
    exactly the bytes the broadcast writes, each owned by one receiver."""
    from connex_b200.parallel.wsync import copy_jobs, job_intervals, split_intervals, split_rounds
    named = random_trainer_weights(CFG, "cpu", dtype=torch.float32, seed=2)
    m = engine_manifest(CFG)
    jobs, _, _ = plan_jobs(CFG, m, named)
    want = set()
    for off, n in job_intervals(jobs):
        want |= set(range(off, off + n, 16))
    for receivers in (1, 3, 7):
        sl = -(-m.total // (receivers * 16)) * 16
        got = []
        for r in split_rounds(jobs, 16):
            for k, ivs in enumerate(split_intervals(job_intervals(r), sl, receivers)):
                for off, n in ivs:
                    assert off >= k * sl and (k == receivers - 1 or off + n <= (k + 1) * sl)
                    got += list(range(off, off + n, 16))
                cj, nt = copy_jobs(ivs, 0)
                assert sum(row[2] * row[3] * 2 for row in cj.tolist()) == sum(n for _, n in ivs)
        assert len(got) == len(set(got)) and set(got) == want


def test_plan_rejects_bad_shapes():
    named = random_trainer_weights(CFG, "cpu")
    named["model.norm.weight"] = torch.ones(CFG.hidden + 8)
    with pytest.raises(ValueError):
        plan_jobs(CFG, engine_manifest(CFG), named)


def test_trainer_layout_covers_engine_params():
    n_tr = sum(torch.Size(s).numel() for _, s in trainer_layout(CFG))
    n_en = sum(torch.Size(s).numel() for _, s in LlamaWeights.layout(CFG))
    assert n_tr == n_en == CFG.num_params()


@pytest.mark.gpu
@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_wsync_kernel_local(dtype):
    from connex_b200 import ops
    from connex_b200.parallel.wsync import apply_local
    dev = torch.device("cuda", 0)
    named = random_trainer_weights(CFG, dev, dtype=dtype, seed=3)
    m = engine_manifest(CFG)
    jobs, _, _ = plan_jobs(CFG, m, named)
    arena = torch.zeros(m.total + 4096, dtype=torch.uint8, device=dev)
    flag = arena.data_ptr() + m.total
    n0 = ops.launch_count()
    ctas = apply_local(jobs, arena[:m.total], flag_addr=flag)
    torch.cuda.synchronize()
    assert ops.launch_count() == n0 + 1
    assert arena[m.total:m.total + 4].view(torch.int32).item() == ctas
    want = _engine_bytes(CFG, fuse_reference(CFG, {k: v.cpu() for k, v in named.items()}), m)
    assert torch.equal(arena[:m.total].cpu(), want)


_CHILD = r"""
import os, sys, json, torch, torch.distributed as dist
from datetime import timedelta
from connex_b200.models.llama import LlamaConfig, random_trainer_weights
from connex_b200.parallel.wsync import WeightBroadcast, fuse_reference, engine_manifest
rank = int(os.environ["RANK"]); dev = torch.device("cuda", int(os.environ["LOCAL_RANK"]))
torch.cuda.set_device(dev)
dist.init_process_group("nccl", device_id=dev, timeout=timedelta(seconds=60))
cfg = LlamaConfig.tiny(layers=2)
bc = WeightBroadcast(cfg, mode=sys.argv[1])
ok = True
for v in (1, 2):
    named = random_trainer_weights(cfg, dev, seed=v) if rank == 0 else None
    bc.sync(named)
    torch.cuda.synchronize(); bc.check()
    ref = fuse_reference(cfg, {k: t.cpu() for k, t in random_trainer_weights(cfg, dev, seed=v).items()})
    if rank != 0:
        for e in bc.manifest.entries:
            got = bc.arena[e.offset:e.offset + e.nbytes].cpu().view(torch.bfloat16).view(e.shape)
            ok &= bool(torch.equal(got, ref[e.name]))
res = [None] * dist.get_world_size()
dist.all_gather_object(res, {"rank": rank, "ok": ok, "mc": bool(bc.mc)})
if rank == 0:
    print(json.dumps(res))
bc.close()
dist.destroy_process_group()
"""


@pytest.mark.gpu
@pytest.mark.parametrize("mode", ["auto", "multicast", "p2p", "relay", "relay_p2p"])
def test_wsync_broadcast_two_gpus(mode, tmp_path):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    script = tmp_path / "child.py"
    script.write_text(_CHILD)
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    env = dict(os.environ, NCCL_DEBUG="WARN", PYTHONPATH=root)
    r = subprocess.run(["timeout", "-k", "10", "180", sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
                        "--nproc-per-node", "2", "--master-addr", "127.0.0.1", "--master-port", "29631", str(script),
                        mode], capture_output=True, text=True, env=env, cwd=root)
    assert r.returncode == 0, r.stderr[-3000:]
    import json
    res = json.loads([ln for ln in r.stdout.splitlines() if ln.startswith("[")][-1])
    assert all(x["ok"] for x in res), res


@pytest.mark.parametrize("world", [2, 3])
def test_sharded_trainers_cover_the_arena_exactly(world):
    """FSDP dim-0 shards on ``world`` trainer ranks: the union of every
    rank's jobs writes the same bytes as one unsharded plan."""
    from connex_b200.parallel.wsync import shard_dim0
    named = random_trainer_weights(CFG, "cpu", dtype=torch.float32, seed=5)
    m = engine_manifest(CFG)
    want = _engine_bytes(CFG, fuse_reference(CFG, named), m)
    got = torch.zeros(m.total, dtype=torch.uint8)
    covered = 0
    for r in range(world):
        local, starts = shard_dim0(named, r, world)
        jobs, _, srcs = plan_jobs(CFG, m, local, task_bytes=4096, starts=starts)
        part = emulate_jobs(jobs, srcs, m.total)
        written = part != 0
        got[written] = part[written]
        covered += sum(t.numel() for t in local.values())
    assert covered == CFG.num_params()
    assert torch.equal(got, want)


def test_shard_start_must_sit_on_a_block():
    from connex_b200.parallel.wsync import plan_jobs as pj
    named = random_trainer_weights(CFG, "cpu")
    g = "model.layers.0.mlp.gate_proj.weight"
    with pytest.raises(ValueError, match="block"):
        pj(CFG, engine_manifest(CFG), {g: named[g][3:]}, starts={g: 3})
    n = "model.norm.weight"
    with pytest.raises(ValueError, match="8-element"):
        pj(CFG, engine_manifest(CFG), {n: named[n][4:]}, starts={n: 4})


def test_nccl_baseline_unpack_matches_the_kernel_layout():
    """The sharded NCCL baseline's receive side (packed bf16 -> engine arena
    with PyTorch strided copies) writes the same bytes as the fused plan."""
    from connex_b200.bench.wsync_bench import unpack_jobs
    from connex_b200.parallel.wsync import shard_dim0
    named = random_trainer_weights(CFG, "cpu", dtype=torch.float32, seed=9)
    m = engine_manifest(CFG)
    got = torch.zeros(m.total, dtype=torch.uint8)
    for r in range(2):
        local, starts = shard_dim0(named, r, 2)
        jobs, _, _ = plan_jobs(CFG, m, local, starts=starts)
        packed = torch.cat([v.to(torch.bfloat16).reshape(-1) for v in local.values()])
        unpack_jobs(jobs, packed, got)
    assert torch.equal(got, _engine_bytes(CFG, fuse_reference(CFG, named), m))
