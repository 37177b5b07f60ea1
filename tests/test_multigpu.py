"""Multi-GPU paths.

CPU part (gloo, world size 2, runs everywhere): the head partition and the
sharing of the NCCL id across ranks.  GPU part (2 GPUs, skipped otherwise):
heads sharded over two ranks + the library's NCCL all-gather must reproduce
the single-GPU result, and a rank that never joins must make the other rank's
communicator creation fail with ANIMAXS_ERR_TIMEOUT instead of hanging.
Failures are made on the host only; NVLS is off in these children.
"""
import os
import socket

import numpy as np
import pytest

from animaxs_b200.sharded import head_range


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_head_partition_covers_all_heads_once():
    for world in (1, 2, 4, 8, 16):
        got = [h for r in range(world) for h in range(*head_range(r, world, 16))]
        assert got == list(range(16))
    from animaxs_b200 import AttentionValidationError
    with pytest.raises(AttentionValidationError):
        head_range(0, 3, 16)
    with pytest.raises(AttentionValidationError):
        head_range(2, 2, 16)


def _gloo_uid_worker(rank, world, port, out):
    import torch.distributed as dist
    from animaxs_b200.sharded import share_unique_id
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank,
                            world_size=world)
    uid = share_unique_id(make_id=lambda: bytes(range(128)))
    out[rank] = uid
    dist.barrier()
    dist.destroy_process_group()


def test_unique_id_is_shared_over_gloo():
    import torch.multiprocessing as mp
    mgr = mp.Manager()
    out = mgr.dict()
    mp.spawn(_gloo_uid_worker, args=(2, _free_port(), out), nprocs=2, join=True)
    assert out[0] == out[1] == bytes(range(128))


# ------------------------------------------------------------------ 2 GPUs --
def _gpu_count():
    try:
        import torch
        return torch.cuda.device_count()
    except Exception:
        return 0


needs2 = pytest.mark.skipif(_gpu_count() < 2, reason="needs 2 GPUs")


def _sharded_worker(rank, world, port, out):
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    import torch
    import torch.distributed as dist

    import animaxs_b200 as ax
    from animaxs_b200.sharded import HeadShardedAttention, share_unique_id
    torch.cuda.set_device(rank)
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank,
                            world_size=world)
    ex = ax.AttentionExecutor(rank)
    uid = share_unique_id()
    sh = HeadShardedAttention(ex, rank, world, uid)
    g = torch.Generator(device="cuda").manual_seed(3)
    results = {}
    for layout in ("token", "head"):
        q, k, v = (torch.randn(1, 2048, 16, 128, generator=g, device="cuda").half() for _ in range(3))
        rope = torch.from_numpy(ax.DitRoPE.generate(1, 32, 64)).cuda()
        if layout == "head":
            o = torch.empty(1, 16, 2048, 128, dtype=torch.float16, device="cuda").permute(0, 2, 1, 3)
        else:
            o = torch.empty_like(q)
        sh(q, k, v, out=o, qk_norm="rms_rope", rope_table=rope)
        ref = ex.attention(q, k, v, qk_norm="rms_rope", rope_table=rope)
        torch.cuda.synchronize()
        results[layout] = float((o.float() - ref.float()).abs().max())
    out[rank] = results
    sh.close()
    dist.barrier()
    dist.destroy_process_group()


@pytest.mark.gpu
@pytest.mark.multigpu
@pytest.mark.timeout(180)
@needs2
def test_head_sharded_matches_single_gpu():
    import torch.multiprocessing as mp
    mgr = mp.Manager()
    out = mgr.dict()
    mp.spawn(_sharded_worker, args=(2, _free_port(), out), nprocs=2, join=True)
    for rank in (0, 1):
        for layout, err in out[rank].items():
            assert err == 0.0, f"rank {rank} {layout}-major output differs by {err}"


def _absent_peer_worker(rank, world, port, out):
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    os.environ["ANIMAXS_NCCL_TIMEOUT_S"] = "5"
    import torch
    import torch.distributed as dist

    import animaxs_b200 as ax
    from animaxs_b200 import AttentionTimeoutError
    from animaxs_b200.sharded import HeadShardedAttention, share_unique_id
    torch.cuda.set_device(rank)
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank,
                            world_size=world)
    ex = ax.AttentionExecutor(rank)
    uid = share_unique_id()
    if rank == 0:
        try:
            HeadShardedAttention(ex, 0, world, uid)
            out[0] = "joined"
        except AttentionTimeoutError:
            out[0] = "timeout"
    # rank 1 never creates its communicator
    dist.barrier()
    dist.destroy_process_group()


@pytest.mark.gpu
@pytest.mark.multigpu
@pytest.mark.timeout(180)
@needs2
def test_rank_that_never_joins_times_out():
    import torch.multiprocessing as mp
    mgr = mp.Manager()
    out = mgr.dict()
    mp.spawn(_absent_peer_worker, args=(2, _free_port(), out), nprocs=2, join=True)
    assert out[0] == "timeout"


def test_config4_prompt_seeds_are_disjoint_across_ranks():
    """Batch sharding: every (prompt, step, block) has its own seed."""
    from oracle.inputs import workload_seed
    seeds = {workload_seed(p, s, b) for p in range(8) for s in range(8) for b in range(28)}
    assert len(seeds) == 8 * 8 * 28
    assert [workload_seed(p, 0, 0) for p in range(8)] == list(range(8))
    assert np.all(np.array(sorted(seeds)) >= 0)
