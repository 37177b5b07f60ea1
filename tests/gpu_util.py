"""Shared helpers for the GPU parity tests (device transfer, tolerance checks)."""
import numpy as np

from oracle import attn_oracle as ora

# after fp16 storage, max-abs 2e-3 and mean-abs 2e-4
# against the fp32 oracle (itself rounded to fp16).
MAX_ABS = 2e-3
MEAN_ABS = 2e-4


def to_dev(x, dtype=None):
    import torch
    t = torch.from_numpy(np.ascontiguousarray(x))
    if dtype is not None:
        t = t.to(dtype)
    return t.cuda()


def run_case(ex, case, rows=None, layout="token"):
    """Run a Case through AttentionExecutor.attention; returns fp32 numpy [B,S,H,D]."""
    import torch
    q, k, v = to_dev(case.q), to_dev(case.k), to_dev(case.v)
    if layout == "head":
        # head-major storage [B, H, S, D] viewed as [B, S, H, D]
        q = q.permute(0, 2, 1, 3).contiguous().permute(0, 2, 1, 3)
        k = k.permute(0, 2, 1, 3).contiguous().permute(0, 2, 1, 3)
        v = v.permute(0, 2, 1, 3).contiguous().permute(0, 2, 1, 3)
    rope = None if case.rope_table is None else to_dev(case.rope_table)
    valid = None
    if case.kv_valid_len is not None and len(set(case.kv_valid_len)) == 1:
        valid = case.kv_valid_len[0]
    out = ex.attention(q, k, v, causal=case.causal, qk_norm=case.qk_norm, rope_table=rope,
                       kv_valid_len=valid)
    torch.cuda.synchronize()
    ex.synchronize()
    out = out.float().cpu().numpy()
    if rows is not None:
        out = out[:, rows]
    return out


def assert_parity(actual, oracle_fp32, max_abs=MAX_ABS, mean_abs=MEAN_ABS, what=""):
    assert np.all(np.isfinite(actual)), f"{what}: non-finite output"
    mx, mn = ora.parity(actual, oracle_fp32)
    assert mx <= max_abs and mn <= mean_abs, f"{what}: max-abs {mx:.3e} mean-abs {mn:.3e}"
    return mx, mn
