"""GPU: the weight streamer (WeightStreamer, WeightStreamer.swift:84-213, and
its two-slot ping-pong in DiTBlockExecutor.swift:222-260), through the C ABI.

Six blocks of W4 projection weights in the reference's pack layout (codes,
fp16 scales, fp16 zeros) are streamed from pinned host memory through two
device slots: block b+1 is copied on a copy stream while block b's projection
runs, and a slot is reloaded only after the projection that read it (its
in-flight mark).  Every projection from a streamed slot must equal the same
projection from resident device weights BIT FOR BIT."""
import numpy as np
import pytest

from oracle import inputs

pytestmark = pytest.mark.gpu

N, K, M = 768, 512, 1024


def _pack(seed):
    """One block's execution range: [codes | scale | zero], 256-byte aligned parts."""
    packed, scale, zero = inputs.quant_weight(seed, N, K, 4)
    parts = [packed.view(np.uint8).ravel(), scale.view(np.uint8).ravel(), zero.view(np.uint8).ravel()]
    offs, off = [], 0
    for p in parts:
        offs.append(off)
        off += (p.size + 255) // 256 * 256
    blob = np.zeros(off, dtype=np.uint8)
    for o, p in zip(offs, parts):
        blob[o:o + p.size] = p
    return blob, offs, (packed, scale, zero)


def test_two_slot_ping_pong_equals_resident_weights():
    import torch

    from animaxs_b200 import AttentionExecutor, ProjectionExecutor, QuantizedWeight, WeightStreamer
    ex = AttentionExecutor(0)
    pj = ProjectionExecutor(ex)
    try:
        blocks = [_pack(100 + b) for b in range(6)]
        size = blocks[0][0].size
        offs = blocks[0][1]
        host = torch.from_numpy(np.concatenate([b[0] for b in blocks])).pin_memory()
        g = torch.Generator(device="cuda").manual_seed(4)
        x = torch.randn(M, K, generator=g, device="cuda").half()
        # resident reference
        ref = []
        for _, _, (packed, scale, zero) in blocks:
            w = QuantizedWeight(*(torch.from_numpy(a).cuda() for a in (packed, scale, zero)), 4, K)
            ref.append(pj.linear(x, w))
        torch.cuda.synchronize()
        ex.synchronize()

        ws = WeightStreamer(ex, capacity=size, slot_count=2)
        copy = torch.cuda.Stream()
        compute = torch.cuda.current_stream()

        def block_src(b):
            return (host.data_ptr() + b * size, size)

        def weight_in(slot):
            return QuantizedWeight(ws.buffer(slot, offs[0], (N, K // 2)),
                                   ws.buffer(slot, offs[1], (N, K // 64), torch.float16),
                                   ws.buffer(slot, offs[2], (N, K // 64), torch.float16), 4, K)
        outs = []
        ws.load(block_src(0), slot=0, logical_index=0, stream=copy)
        for b in range(len(blocks)):
            slot = b % 2
            if b + 1 < len(blocks):
                # into the other slot, ordered after block b-1's projection (its mark)
                ws.load(block_src(b + 1), slot=(b + 1) % 2, logical_index=b + 1, stream=copy)
            ws.wait_loaded(slot, compute)
            outs.append(pj.linear(x, weight_in(slot)))
            ws.mark_in_flight(slot, compute)
        torch.cuda.synchronize()
        ex.synchronize()
        for b, (o, r) in enumerate(zip(outs, ref)):
            a, e = o.cpu().numpy().view(np.uint16), r.cpu().numpy().view(np.uint16)
            assert np.array_equal(a, e), f"block {b}: {np.count_nonzero(a != e)} outputs differ"
        assert ws.loaded_logical_indexes == [4, 5]
        assert ws.in_flight_slot_set == {0, 1}
        ws.complete(0)
        assert ws.in_flight_slot_set == {1}
        ws.close()
    finally:
        ex.close()


def test_streamer_refuses_what_the_reference_refuses():
    import torch

    from animaxs_b200 import AttentionExecutor, AttentionValidationError, WeightStreamer
    ex = AttentionExecutor(0)
    try:
        with pytest.raises(AttentionValidationError, match="capacity must be positive"):
            WeightStreamer(ex, capacity=0)
        with pytest.raises(AttentionValidationError, match="slot count must be in 1...4"):
            WeightStreamer(ex, capacity=1024, slot_count=5)
        ws = WeightStreamer(ex, capacity=1024, slot_count=1)
        src = torch.zeros(2048, dtype=torch.uint8).pin_memory()
        with pytest.raises(AttentionValidationError, match="does not fit the weight slot"):
            ws.load(src)
        with pytest.raises(AttentionValidationError, match="out of range"):
            ws.load(src[:512], slot=1)
        ws.load(src[:1024], logical_index=7)
        torch.cuda.synchronize()
        assert ws.loaded_logical_indexes == [7]
        assert bool((ws.buffer(0) == 0).all())
        ws.close()
    finally:
        ex.close()
