"""Multi-GPU paths.

CPU part (gloo, world size 2, runs everywhere):
* the head partition;
* the sharing of the NCCL id and of the IPC handles across ranks.

GPU part (2 GPUs, skipped otherwise):
* Heads sharded over two ranks must reproduce the single-GPU result bit for
  bit, both with the library's NCCL all-gather and with the fused peer path,
  where the attention kernel stores every tile into both ranks' outputs over
  NVLink.
* A rank that never joins must make the other rank fail with
  ANIMAXS_ERR_TIMEOUT instead of hanging. For NCCL that is communicator
  creation; for the peer path, the bounded handshake waits.

Failures are made on the host only (a rank that does not call).  NVLS is off
in these children and no kernel uses multimem.
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
    mgr = mp.get_context("spawn").Manager()
    out = mgr.dict()
    mp.spawn(_gloo_uid_worker, args=(2, _free_port(), out), nprocs=2, join=True)
    assert out[0] == out[1] == bytes(range(128))


def _gloo_handles_worker(rank, world, port, out):
    import torch.distributed as dist
    from animaxs_b200.sharded import exchange_handles
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank,
                            world_size=world)
    out[rank] = exchange_handles(bytes([rank]) * 64)
    dist.barrier()
    dist.destroy_process_group()


def test_ipc_handles_are_exchanged_in_rank_order_over_gloo():
    import torch.multiprocessing as mp
    mgr = mp.get_context("spawn").Manager()
    out = mgr.dict()
    mp.spawn(_gloo_handles_worker, args=(2, _free_port(), out), nprocs=2, join=True)
    want = bytes([0]) * 64 + bytes([1]) * 64
    assert out[0] == out[1] == want


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
    mgr = mp.get_context("spawn").Manager()
    out = mgr.dict()
    mp.spawn(_sharded_worker, args=(2, _free_port(), out), nprocs=2, join=True)
    for rank in (0, 1):
        for layout, err in out[rank].items():
            assert err == 0.0, f"rank {rank} {layout}-major output differs by {err}"


def _absent_peer_worker(rank, world, port, out, one_gpu=False):
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    os.environ["ANIMAXS_NCCL_TIMEOUT_S"] = "5"
    import torch
    import torch.distributed as dist

    import animaxs_b200 as ax
    from animaxs_b200 import AttentionTimeoutError
    from animaxs_b200.sharded import HeadShardedAttention, share_unique_id
    device = 0 if one_gpu else rank
    torch.cuda.set_device(device)
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank,
                            world_size=world)
    ex = ax.AttentionExecutor(device)
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
    mgr = mp.get_context("spawn").Manager()
    out = mgr.dict()
    mp.spawn(_absent_peer_worker, args=(2, _free_port(), out), nprocs=2, join=True)
    assert out[0] == "timeout"


@pytest.mark.gpu
@pytest.mark.timeout(180)
def test_rank_that_never_joins_times_out_on_one_gpu():
    """The communicator deadline with both ranks as processes on one GPU:
    rank 1 never creates its communicator, so rank 0's non-blocking NCCL
    initialisation waits in the bootstrap (no kernel runs) until the 5 s
    deadline and reports the timeout."""
    import torch.multiprocessing as mp
    mgr = mp.get_context("spawn").Manager()
    out = mgr.dict()
    mp.spawn(_absent_peer_worker, args=(2, _free_port(), out, True), nprocs=2, join=True)
    assert out[0] == "timeout"


def _peer_worker(rank, world, port, out):
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    import torch
    import torch.distributed as dist

    import animaxs_b200 as ax
    from animaxs_b200.sharded import PeerShardedAttention
    torch.cuda.set_device(rank)
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank,
                            world_size=world)
    ex = ax.AttentionExecutor(rank)
    s_len = 2048
    ps = PeerShardedAttention(ex, rank, world, (1, s_len, 16, 128))
    g = torch.Generator(device="cuda").manual_seed(5)   # the same inputs on both ranks
    rope = torch.from_numpy(ax.DitRoPE.generate(1, 32, 64)).cuda()
    errs = []
    for call in range(3):   # repeated calls: the handshake words advance per call
        q, k, v = (torch.randn(1, s_len, 16, 128, generator=g, device="cuda").half() for _ in range(3))
        got = ps(q, k, v, qk_norm="rms_rope", rope_table=rope) if call != 1 else ps(q, k, v)
        ex.synchronize()
        ref = ex.attention(q, k, v, qk_norm="rms_rope", rope_table=rope) if call != 1 else ex.attention(q, k, v)
        torch.cuda.synchronize()
        errs.append(float((got.float() - ref.float()).abs().max()))
        dist.barrier()   # the next call may overwrite the output
    ps.close()
    # Head-major output, GQA (16 query heads over 4 K/V heads), causal.
    ps = PeerShardedAttention(ex, rank, world, (1, 1000, 16, 128), layout="head")
    q = torch.randn(1, 1000, 16, 128, generator=g, device="cuda").half()
    k, v = (torch.randn(1, 1000, 4, 128, generator=g, device="cuda").half() for _ in range(2))
    got = ps(q, k, v, causal=True)
    ex.synchronize()
    ref = ex.attention(q, k, v, causal=True)
    torch.cuda.synchronize()
    errs.append(float((got.float() - ref.float()).abs().max()))
    dist.barrier()
    ps.close()
    # head_dim 64 (the LLM adapter's heads), 2 images, fused RMSNorm + RoPE.
    ps = PeerShardedAttention(ex, rank, world, (2, 512, 16, 64))
    tab = torch.from_numpy(ax.adapter_rope(512)).cuda()
    q, k, v = (torch.randn(2, 512, 16, 64, generator=g, device="cuda").half() for _ in range(3))
    got = ps(q, k, v, qk_norm="rms_rope", rope_table=tab)
    ex.synchronize()
    ref = ex.attention(q, k, v, qk_norm="rms_rope", rope_table=tab)
    torch.cuda.synchronize()
    errs.append(float((got.float() - ref.float()).abs().max()))
    dist.barrier()
    ps.close()
    # 4096 tokens: 8 heads x 16 pairs = 128 pairs per rank leave SMs idle, so
    # the launch deals 256 single tiles -- more than one per CTA, the per-rank
    # shape of 16K tokens over 8 ranks.  Two calls in a row.
    ps = PeerShardedAttention(ex, rank, world, (1, 4096, 16, 128))
    rope = torch.from_numpy(ax.DitRoPE.generate(1, 64, 64)).cuda()
    for call in range(2):
        q, k, v = (torch.randn(1, 4096, 16, 128, generator=g, device="cuda").half() for _ in range(3))
        got = ps(q, k, v, qk_norm="rms_rope", rope_table=rope)
        ex.synchronize()
        ref = ex.attention(q, k, v, qk_norm="rms_rope", rope_table=rope)
        torch.cuda.synchronize()
        errs.append(float((got.float() - ref.float()).abs().max()))
        dist.barrier()
    ps.close()
    out[rank] = errs
    dist.barrier()
    dist.destroy_process_group()


@pytest.mark.gpu
@pytest.mark.multigpu
@pytest.mark.timeout(180)
@needs2
def test_peer_fused_head_sharded_matches_single_gpu():
    """The attention kernel stores its heads into both ranks' outputs (NVLink);
    every rank's buffer equals the single-GPU result bit for bit: three calls
    in a row (token-major, norm + RoPE and plain), a head-major GQA causal
    call with a ragged length, head_dim 64 over two images, and two calls at
    4096 tokens whose 256 single-tile items are more than one per CTA."""
    import torch.multiprocessing as mp
    mgr = mp.get_context("spawn").Manager()
    out = mgr.dict()
    mp.spawn(_peer_worker, args=(2, _free_port(), out), nprocs=2, join=True)
    for rank in (0, 1):
        assert out[rank] == [0.0] * 7, f"rank {rank}: max differences {out[rank]}"


def _peer_absent_worker(rank, world, port, out, one_gpu=False):
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    import torch
    import torch.distributed as dist

    import animaxs_b200 as ax
    from animaxs_b200 import AttentionTimeoutError
    from animaxs_b200.sharded import PeerShardedAttention
    device = 0 if one_gpu else rank
    torch.cuda.set_device(device)
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank,
                            world_size=world)
    ex = ax.AttentionExecutor(device)
    ps = PeerShardedAttention(ex, rank, world, (1, 512, 16, 128))
    if rank == 1:
        # A sentinel in rank 1's output: rank 0's call must not store into a
        # peer whose readiness it never saw.
        ps.output.fill_(7.0)
        torch.cuda.synchronize()
    dist.barrier()
    if rank == 0:
        # Rank 1 stays alive but never calls: both bounded waits of this call
        # give up (2 s each) and the status word reports the timeout.
        g = torch.Generator(device="cuda").manual_seed(1)
        q, k, v = (torch.randn(1, 512, 16, 128, generator=g, device="cuda").half() for _ in range(3))
        ps(q, k, v)
        try:
            ex.synchronize()
            out[0] = "completed"
        except AttentionTimeoutError:
            out[0] = "timeout"
        # the context still works after the report
        ref = ex.attention(q, k, v)
        ex.synchronize()
        out["after"] = bool(torch.isfinite(ref.float()).all())
    dist.barrier()   # rank 1 leaves only after rank 0's kernels have finished
    if rank == 1:
        torch.cuda.synchronize()
        out["untouched"] = bool((ps.output == 7.0).all())
    ps.close()
    dist.barrier()
    dist.destroy_process_group()


@pytest.mark.gpu
@pytest.mark.multigpu
@pytest.mark.timeout(180)
@needs2
def test_peer_that_never_calls_times_out():
    import torch.multiprocessing as mp
    mgr = mp.get_context("spawn").Manager()
    out = mgr.dict()
    mp.spawn(_peer_absent_worker, args=(2, _free_port(), out), nprocs=2, join=True)
    assert out[0] == "timeout" and out["after"]
    assert out["untouched"], "rank 0 stored into rank 1's output after its ready handshake timed out"


@pytest.mark.gpu
@pytest.mark.timeout(180)
def test_peer_that_never_calls_times_out_on_one_gpu():
    """The same failure with both ranks as processes on one GPU (CUDA IPC
    maps a buffer of the same device into the other process).  Rank 1 never
    launches anything, so rank 0's bounded waits are the only kernels that
    wait: the opening handshake gives up after 2 s, the attention kernel
    stores nothing into rank 1's buffer and adds no arrival, the closing wait
    gives up, synchronize reports the timeout and the context keeps working."""
    import torch.multiprocessing as mp
    mgr = mp.get_context("spawn").Manager()
    out = mgr.dict()
    mp.spawn(_peer_absent_worker, args=(2, _free_port(), out, True), nprocs=2, join=True)
    assert out[0] == "timeout" and out["after"]
    assert out["untouched"], "rank 0 stored into rank 1's output after its ready handshake timed out"


def test_peer_sharded_rejects_bad_shape_before_touching_a_device():
    """PeerShardedAttention checks its output shape and layout before any
    library or device call."""
    from animaxs_b200 import AttentionValidationError
    from animaxs_b200.sharded import PeerShardedAttention

    class NoDevice:
        handle = None
        device = 0

        def last_error(self):
            return ""
    with pytest.raises(AttentionValidationError):
        PeerShardedAttention(NoDevice(), 0, 2, (1, 2, 3))
    with pytest.raises(AttentionValidationError):
        PeerShardedAttention(NoDevice(), 0, 2, (1, 8, 2, 64), layout="diagonal")


def test_config4_prompt_seeds_are_disjoint_across_ranks():
    """Batch sharding: every (prompt, step, block) has its own seed."""
    from oracle.inputs import workload_seed
    seeds = {workload_seed(p, s, b) for p in range(8) for s in range(8) for b in range(28)}
    assert len(seeds) == 8 * 8 * 28
    assert [workload_seed(p, 0, 0) for p in range(8)] == list(range(8))
    assert np.all(np.array(sorted(seeds)) >= 0)
