"""Generate the golden fixtures in this directory from the REFERENCE's own oracles.

Run once, in a container where the AnimaXS source tree is present:

    python tests/golden/make_golden.py --reference <path-to-AnimaXS-checkout>

It imports the reference's PyTorch CPU oracles
(``scripts/dit_source_oracle.py`` and ``scripts/qwen_comfy_oracle.py``) and
calls their functions -- ``rms_norm``, ``dit_rope``, ``apply_split_half_rope``,
``scaled_dot_product``, ``precompute_freqs_cis``, ``apply_rope``,
``attention_pytorch`` -- on seeded inputs, then writes small ``.npz`` files:

* ``rope_tables.npz``   -- sampled rows + full-table checksums of the 3-D RoPE
  tables for the 32x32 / 64x64 / 128x128 grids, the reference's committed
  ``scripts/oracle_out/dit_rope_oracle.npz`` (sampled rows), and the Qwen
  1-D table (theta 1e6).
* ``attn_small.npz``    -- complete outputs of small cases (DiT self with
  rms+rope3d, DiT cross with rms and with/without a key-padding mask, Qwen
  GQA prefill with causal + padding masks).
* ``attn_configs.npz``  -- outputs at sampled query rows for the benchmark
  configurations 1, 2, 3 (layers 0 and 27), 4 (a subset of blocks) and 5.
* ``proj_small.npz``    -- the fused projections (q|k|v with RMSNorm and
  RoPE, and the out-projection's gated residual) through ``linear``,
  ``rms_norm``, ``dit_rope`` and ``apply_split_half_rope``.
* ``real_context.npz``  -- real activations from the reference's committed
  ``scripts/oracle_out/adapter_oracle_case1.npz`` (an actual prompt run
  through the model): the LLM adapter's block-0 hidden state [47, 1024]
  (magnitudes up to 64) and the 47 valid rows of the 512-row padded context
  the DiT cross-attention reads, stored as fp16.  Used as realistic attention
  inputs (heavy-tailed values, a context padded with zero rows).
* ``quant_small.npz``   -- W8 / W4 weights packed by the reference's own
  quantizer (``scripts/pack_anima.py`` ``_quantize_chunk``, plain and with the
  W4 range search) and decoded by its own decoders
  (``scripts/animapk_cuda/quant.py`` ``decode_w8_matrix`` /
  ``decode_w4_matrix``), with ragged groups and odd packed rows, plus one
  projection through ``linear`` with the decoded W4 weight.  The packed bytes,
  scales and zeros are stored verbatim: they are the kernels' inputs.

Only the inputs' seeds are stored (plus checksums of the inputs to detect a
change in ``torch.Generator``); tests regenerate inputs with
``oracle/inputs.py``.  Nothing here is imported at test time -- the tests
read the ``.npz`` files only.
"""

from __future__ import annotations

import argparse
import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))
from oracle import inputs  # noqa: E402  (seeded input generator only)

SAMPLE_ROWS = [0, 1, 2, 3, 5, 8, 31, 63, 64, 127, 128, 129, 200, 255, 256, 298, 299,
               300, 301, 383, 384, 511, 512, 1000, 1023, 1024, 2047, 2048, 3000, 4095,
               4096, 8191, 8192, 12345, 16383]


def sample_rows(n: int) -> np.ndarray:
    return np.array(sorted({r for r in SAMPLE_ROWS if r < n}), dtype=np.int64)


def checksum(x) -> np.ndarray:
    x = np.asarray(x, dtype=np.float64)
    return np.array([x.sum(), np.abs(x).sum(), (x * x).sum()], dtype=np.float64)


def load_reference(path: str):
    sys.path.insert(0, os.path.join(path, "scripts"))
    import dit_source_oracle as dso  # noqa: E402
    import qwen_comfy_oracle as qco  # noqa: E402
    return dso, qco


def t32(x):
    return torch.from_numpy(np.asarray(x, dtype=np.float32))


def ref_dit(dso, case, rows):
    """DiT path: rms_norm -> (apply_split_half_rope) -> scaled_dot_product, fp32."""
    q, k, v = t32(case.q), t32(case.k), t32(case.v)
    ones = torch.ones(128, dtype=torch.float32)
    qn, kn = dso.rms_norm(q, ones), dso.rms_norm(k, ones)
    if case.qk_norm == "rms_rope":
        qn, kn = dso.apply_split_half_rope(qn, kn, t32(case.rope_table))
    if case.kv_valid_len is None:
        outs = []
        for h in range(q.shape[2]):  # per head: scaled_dot_product holds all scores
            outs.append(dso.scaled_dot_product(qn[:, rows, h:h + 1], kn[:, :, h:h + 1],
                                               v[:, :, h:h + 1]))
        return torch.cat(outs, dim=2).numpy()
    return ref_masked(case, qn, kn, v, rows, causal=False)


def ref_masked(case, qn, kn, v, rows, causal):
    """Masked SDPA through the reference's attention_pytorch (additive mask)."""
    _, qco = REF
    b, sq, hq, d = qn.shape
    sk, hkv = kn.shape[1], kn.shape[2]
    valid = case.kv_valid_len[0] if case.kv_valid_len else sk
    # QwenOracle.forward mask construction (qwen_comfy_oracle.py:238-248)
    am = torch.zeros(1, sk)
    am[:, :valid] = 1.0
    mask = 1.0 - am.reshape(1, 1, -1, sk).expand(1, 1, sq, sk)
    mask = mask.masked_fill(mask.to(torch.bool), torch.finfo(torch.float32).min / 4)
    if causal:
        cm = torch.empty(sq, sk).fill_(torch.finfo(torch.float32).min / 4).triu_(1)
        mask = mask + cm
    mask = mask[:, :, rows, :].reshape(1, len(rows), sk)
    xq = qn[:, rows].transpose(1, 2)
    xk = kn.transpose(1, 2)
    xv = v.transpose(1, 2)
    out = qco.attention_pytorch(xq, xk, xv, hq, mask=mask, skip_reshape=True,
                                enable_gqa=(hq != hkv))
    return out.reshape(b, len(rows), hq, d).numpy()


def ref_qwen(case, rows):
    """Qwen path: rms_norm -> precompute_freqs_cis/apply_rope -> attention_pytorch."""
    _, qco = REF
    q, k, v = t32(case.q), t32(case.k), t32(case.v)
    s = q.shape[1]
    ones = torch.ones(128, dtype=torch.float32)
    xq = qco.rms_norm(q.transpose(1, 2), ones, 1e-6)
    xk = qco.rms_norm(k.transpose(1, 2), ones, 1e-6)
    pos = torch.arange(0, s).unsqueeze(0)
    freqs = qco.precompute_freqs_cis(128, pos, 1.0e6)
    xq, xk = qco.apply_rope(xq, xk, freqs)
    return ref_masked(case, xq.transpose(1, 2), xk.transpose(1, 2), v, rows, causal=True)


def make_proj(dso):
    """``proj_small.npz``: the fused projections through the reference's own
    ``linear`` (fp32 matmul cast to fp16), ``rms_norm`` (fp32 in and out, no
    rounding between norm and rotation, as the fused Metal kernel),
    ``dit_rope`` and ``apply_split_half_rope``, and the block's gated residual
    update ``x + gate * out`` (fp32 residual, fp16 branch)."""
    out = {}
    images, tokens = 2, 64
    x, w, qw, kw = inputs.proj_qkv(seed=21, images=images, tokens=tokens, k=256, q_heads=2, k_heads=2,
                                   v_cols=256)
    y = dso.linear(torch.from_numpy(x), torch.from_numpy(w))          # fp16 [128, 768]
    m = y.shape[0]
    q = y[:, :256].float().reshape(images, tokens, 2, 128)
    k = y[:, 256:512].float().reshape(images, tokens, 2, 128)
    qn = dso.rms_norm(q, torch.from_numpy(qw).float())
    kn = dso.rms_norm(k, torch.from_numpy(kw).float())
    rope = dso.dit_rope(8, 8, 1)                                       # 64 tokens
    qr, kr = dso.apply_split_half_rope(qn, kn, rope)
    v = y[:, 512:].float()
    out["qkv_rope_out"] = torch.cat([qr.reshape(m, 256), kr.reshape(m, 256), v], dim=1).numpy()
    out["qkv_rms_out"] = torch.cat([qn.reshape(m, 256), kn.reshape(m, 256), v], dim=1).numpy()
    out["qkv_in_checksum"] = np.concatenate([checksum(x), checksum(w), checksum(qw), checksum(kw)])
    out["qkv_meta"] = np.array([21, images, tokens, 256, 2, 2, 256], dtype=np.int64)
    xg, wg, res, gate = inputs.proj_gate(seed=22, images=images, tokens=tokens, k=256, n=256)
    branch = dso.linear(torch.from_numpy(xg), torch.from_numpy(wg)).float()
    g = torch.from_numpy(gate)[torch.arange(m) // tokens]
    out["gate_out"] = (torch.from_numpy(res) + g * branch).numpy()
    out["gate_in_checksum"] = np.concatenate([checksum(xg), checksum(wg), checksum(res), checksum(gate)])
    out["gate_meta"] = np.array([22, images, tokens, 256, 256], dtype=np.int64)
    np.savez_compressed(os.path.join(HERE, "proj_small.npz"), **out)


def make_quant(dso, path):
    """``quant_small.npz`` (see the module docstring)."""
    sys.path.insert(0, os.path.join(path, "scripts"))
    import pack_anima  # noqa: E402
    from animapk_cuda import quant  # noqa: E402
    out = {}
    cases = [("w8", 8, 40, 200, False, 31), ("w4", 4, 40, 200, False, 32),
             ("w4opt", 4, 33, 129, True, 33), ("w4wide", 4, 64, 1024, True, 34)]
    for name, bits, rows, k, opt, seed in cases:
        g = torch.Generator().manual_seed(seed)
        chunk = (torch.randn(rows, k, generator=g) * 0.04).numpy().astype(np.float32)
        chunk[0, 3] = 0.5                       # an outlier stretches one group's range
        chunk[1, :64] = 0.125                   # a constant group (span < 1e-8: scale 1)
        data, sc, ze, _ = pack_anima._quantize_chunk(chunk, bits, 64, opt)
        dec = quant.decode_w4_matrix(data, sc, ze, rows, k) if bits == 4 else \
            quant.decode_w8_matrix(data, sc, ze, rows, k)
        groups = (k + 63) // 64
        out[name + "_packed"] = np.frombuffer(data, dtype=np.uint8).reshape(rows, -1)
        out[name + "_scale"] = np.frombuffer(sc, dtype="<f2").reshape(rows, groups)
        out[name + "_zero"] = np.frombuffer(ze, dtype="<f2").reshape(rows, groups)
        out[name + "_decoded_f32"] = dec.numpy().astype(np.float32)
        out[name + "_decoded_half"] = dec.half().numpy()
        out[name + "_meta"] = np.array([bits, rows, k, int(opt), seed], dtype=np.int64)
    # A projection with the decoded W4 weight (the dequantize-then-GEMM path of
    # LinearExecutor.swift:153-189) through the reference's linear.
    x = torch.from_numpy(inputs.proj_x(35, 64, 1024))
    wdec = torch.from_numpy(out["w4wide_decoded_half"])
    out["proj_w4_out"] = dso.linear(x, wdec).float().numpy()
    out["proj_w4_meta"] = np.array([35, 64, 1024], dtype=np.int64)
    np.savez_compressed(os.path.join(HERE, "quant_small.npz"), **out)


def make_real_context(path):
    """``real_context.npz`` (see the module docstring)."""
    z = np.load(os.path.join(path, "scripts/oracle_out/adapter_oracle_case1.npz"))
    ctx = z["adapter_out_padded512"][0]
    valid = int((np.abs(ctx).sum(axis=1) > 0).sum())
    assert not np.abs(ctx[valid:]).any(), "padding rows are expected to be zero"
    out = {
        "hidden": z["adapter_block_00"][0].astype(np.float16),
        "context_valid": ctx[:valid].astype(np.float16),
        "context_rows": np.array([ctx.shape[0], valid], dtype=np.int64),
        "source_commit": np.array(str(z["commit"])),
    }
    np.savez_compressed(os.path.join(HERE, "real_context.npz"), **out)


def main():
    global REF
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True, help="AnimaXS source checkout")
    ap.add_argument("--skip-large", action="store_true")
    ap.add_argument("--only-proj", action="store_true",
                    help="write proj_small.npz, quant_small.npz and real_context.npz only")
    args = ap.parse_args()
    REF = load_reference(args.reference)
    dso, qco = REF
    torch.set_num_threads(os.cpu_count())
    make_proj(dso)
    make_quant(dso, args.reference)
    make_real_context(args.reference)
    if args.only_proj:
        return

    # ---------------- RoPE tables ----------------
    rope = {}
    for (t, h, w) in [(1, 32, 32), (1, 64, 64), (1, 128, 128)]:
        tab = dso.dit_rope(h, w, t).numpy()
        rows = sample_rows(tab.shape[0])
        key = f"rope3d_{t}x{h}x{w}"
        rope[key + "_rows"] = rows
        rope[key + "_sample"] = tab[rows]
        rope[key + "_checksum"] = checksum(tab)
    committed = np.load(os.path.join(args.reference, "scripts/oracle_out/dit_rope_oracle.npz"))
    rows = sample_rows(committed["rope"].shape[0])
    rope["committed_rope_rows"] = rows
    rope["committed_rope_sample"] = committed["rope"][rows]
    rope["committed_rope_checksum"] = checksum(committed["rope"])
    cos, sin, nsin = qco.precompute_freqs_cis(128, torch.arange(0, 512).unsqueeze(0), 1.0e6)
    cos = cos.reshape(512, 128).numpy()
    sin = sin.reshape(512, 64).numpy()
    nsin = nsin.reshape(512, 64).numpy()
    rows = sample_rows(512)
    rope["rope1d_512_rows"] = rows
    rope["rope1d_512_cos"] = cos[rows, :64]
    rope["rope1d_512_sin"] = sin[rows]
    rope["rope1d_512_nsin"] = nsin[rows]
    rope["rope1d_512_checksum"] = checksum(np.concatenate([cos[:, :64], sin], axis=1))
    np.savez_compressed(os.path.join(HERE, "rope_tables.npz"), **rope)

    # ---------------- small complete cases ----------------
    small = {}

    def add(name, case, out, seed_info):
        small[name + "_out"] = out.astype(np.float32)
        small[name + "_in_checksum"] = np.concatenate([checksum(case.q), checksum(case.k),
                                                       checksum(case.v)])
        small[name + "_meta"] = np.array(seed_info, dtype=np.int64)

    c = inputs.dit_self(seed=10, grid=(1, 16, 16), heads=2)
    add("dit_self_256", c, ref_dit(dso, c, np.arange(256)), [10, 1, 16, 16, 2])
    c = inputs.dit_cross(seed=11, q_len=192, kv_len=96, heads=2, kv_valid=40)
    add("dit_cross_192x96_valid40", c, ref_dit(dso, c, np.arange(192)), [11, 192, 96, 2, 40])
    c = inputs.dit_cross(seed=12, q_len=130, kv_len=200, heads=2, kv_valid=None)
    add("dit_cross_130x200", c, ref_dit(dso, c, np.arange(130)), [12, 130, 200, 2, 0])
    c = inputs.qwen_prefill(layer=0, seq_len=160, heads=4, kv_heads=2, valid=100)
    add("qwen_160_h4kv2_valid100", c, ref_qwen(c, np.arange(160)), [0, 160, 4, 2, 100])
    np.savez_compressed(os.path.join(HERE, "attn_small.npz"), **small)

    if args.skip_large:
        return
    # ---------------- benchmark configurations at sampled rows ----------------
    big = {}

    def addbig(name, case, out, rows):
        big[name + "_rows"] = rows
        big[name + "_out"] = out.astype(np.float32)
        big[name + "_in_checksum"] = np.concatenate([checksum(case.q), checksum(case.k),
                                                     checksum(case.v)])

    c = inputs.dit_self(seed=0, grid=(1, 32, 32))
    rows = sample_rows(1024)
    addbig("cfg1", c, ref_dit(dso, c, rows), rows)
    c = inputs.dit_cross(seed=0)
    rows = sample_rows(4096)
    addbig("cfg2_masked", c, ref_dit(dso, c, rows), rows)
    c.kv_valid_len = None
    addbig("cfg2_unmasked", c, ref_dit(dso, c, rows), rows)
    for layer in (0, 27):
        c = inputs.qwen_prefill(layer=layer)
        rows = sample_rows(512)
        addbig(f"cfg3_l{layer}", c, ref_qwen(c, rows), rows)
    for prompt in (0, 7):
        for step in (0, 7):
            for block in (0, 27):
                sc, cc = inputs.workload_block(prompt, step, block)
                rows = sample_rows(4096)[::3]
                tag = f"cfg4_p{prompt}_s{step}_b{block}"
                addbig(tag + "_self", sc, ref_dit(dso, sc, rows), rows)
                addbig(tag + "_cross", cc, ref_dit(dso, cc, rows), rows)
    c = inputs.dit_self(seed=0, grid=(1, 128, 128))
    rows = sample_rows(16384)
    addbig("cfg5", c, ref_dit(dso, c, rows), rows)
    np.savez_compressed(os.path.join(HERE, "attn_configs.npz"), **big)


REF = None

if __name__ == "__main__":
    main()
