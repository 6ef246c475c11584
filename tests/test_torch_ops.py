"""The torch custom-op layer (``torch.ops.lrkv_b200``): every kernel entry point registered with a fake
implementation, so that it traces on meta / fake tensors (``torch.compile``) and refuses CPU tensors; on the GPU the
backend's decode forward compiled with ``fullgraph=True`` gives the eager output bit for bit."""

import pytest
import torch

from belt_b200 import decode as dec
from belt_b200 import latent_ops, ops

META = "meta"


def _bf(*shape):
    return torch.empty(*shape, dtype=torch.bfloat16, device=META)


def _i32(*shape):
    return torch.empty(*shape, dtype=torch.int32, device=META)


def test_every_op_is_registered():
    for name in ops.OPS:
        assert hasattr(torch.ops.lrkv_b200, name), name


def test_ops_trace_on_meta_tensors():
    T, G, nb, page, W = 5, 4, 40, 16, 1024
    segs = [0, 128, 0, 0, 128, 128, 0, 0, 256, 128, 0, 0, 384, 128, 0, 0]
    cache = _bf(nb, 1, page, W)[:, 0]
    torch.ops.lrkv_b200.cache_write(_bf(T, W), torch.empty(T, dtype=torch.int64, device=META), cache, _bf(512, 1024),
                                    segs, 1e-6)
    torch.ops.lrkv_b200.proj_cache_write(_bf(T, 256), _bf(W, 256), _i32(T), cache, _bf(512, 1024), segs, 1e-6)
    sched = dec.DecodeSchedule(148, _i32(T + 148, 4), _i32(149), _i32(T + 1), 10)
    torch.ops.lrkv_b200.decode_schedule(_i32(T), sched.work, sched.cta_seg, sched.seg_base, 148, 1, 10)
    q_bd = torch.ops.lrkv_b200.block_diag_query(_bf(T, 24, 256), _bf(4, 256, 768), [0, 768] + [0, 0] * 11)
    assert q_bd.shape == (T, 24, 768) and q_bd.device.type == META and q_bd.dtype == torch.bfloat16
    part = torch.empty(T + 148, 24, 513, device=META)
    torch.ops.lrkv_b200.latent_decode(q_bd, cache, _i32(T, 8), _i32(T), sched.work, sched.cta_seg, part, 148, 0.0625,
                                      512, 512, [0, 64, 128, 64, 256, 64, 384, 64], _bf(1, 64, 256), _bf(4096, 64))
    a = _bf(T, 24, 512)
    torch.ops.lrkv_b200.merge_segments(part, sched.seg_base, a, torch.empty(T, 24, device=META))
    torch.ops.lrkv_b200.up_project(a, _bf(4, 512, 256), _bf(T, 24, 256))
    torch.ops.lrkv_b200.decompress(cache, _i32(8), 100, 0, _bf(4, 256, 512), segs, _bf(4, 512, 256), 512,
                                   _bf(4096, 64), _bf(100, 4, 256), _bf(100, 4, 256))
    torch.ops.lrkv_b200.prefill_attention(_bf(7, 24, 256), _bf(100, 4, 256), _bf(100, 4, 256), 93, 0, 0.0625, True,
                                          _bf(7, 24, 256), torch.empty(7, 24, device=META))


def test_python_surface_traces_under_compile_on_meta():
    """The package's operator functions (argument checks, then the ops) compile into one graph on meta tensors."""
    from belt_b200.decode import RopeRebuild

    def step(q, qmap, cache, bt, seq_lens, work, cta_seg, seg_base, part, a, lse, v_up, out, blocks, cos_sin):
        sched = dec.DecodeSchedule(148, work, cta_seg, seg_base, 10)
        q_bd = latent_ops.block_diag_query(q, qmap)
        dec.latent_decode(q_bd, cache, bt, seq_lens, sched, part, 0.0625, 512, 512,
                          rope=RopeRebuild(((0, 64), (128, 64), (256, 64), (384, 64)), blocks, cos_sin))
        dec.merge_segments(part, sched, a, lse)
        latent_ops.up_project(a, v_up, out)
        return out

    B = 3
    args = (_bf(B, 24, 256), _bf(4, 256, 768), _bf(20, 1, 16, 1024)[:, 0], _i32(B, 8), _i32(B), _i32(B + 148, 4),
            _i32(149), _i32(B + 1), torch.empty(B + 148, 24, 513, device=META), _bf(B, 24, 512),
            torch.empty(B, 24, device=META), _bf(4, 512, 256), _bf(B, 24, 256), _bf(1, 64, 256), _bf(4096, 64))
    compiled = torch.compile(step, backend="aot_eager", fullgraph=True)
    out = compiled(*args)
    assert out.shape == (B, 24, 256) and out.device.type == META


def test_ops_refuse_cpu_tensors():
    with pytest.raises(NotImplementedError):
        torch.ops.lrkv_b200.block_diag_query(torch.zeros(1, 24, 256, dtype=torch.bfloat16),
                                             torch.zeros(4, 256, 768, dtype=torch.bfloat16), [0, 768] + [0, 0] * 11)


@pytest.mark.gpu
def test_backend_forward_compiles_fullgraph_and_matches_eager():
    """``LatentAttentionImpl.forward`` (cache write of this step's rows, absorbed query, split-KV decode, merge, U_v
    projection) under ``torch.compile(fullgraph=True)``: one graph of the custom ops, the same bits as eager."""
    import oracle
    from belt_b200 import synth
    from belt_b200.latent_backend import (CommonAttentionMetadata, LatentAttentionImpl,
                                          LatentAttentionMetadataBuilder, LatentKVSpec)
    from belt_b200.layer import derive_latent_tensors
    dev = torch.device("cuda", 0)
    w = synth.make_layer(synth.spec_from_ranks(448, 576))
    lat = derive_latent_tensors(w.k_up, w.v_up, w.k_norm_weight, w.layout, synth.cos_sin_table(4096), device=dev)
    seqs = [40, 300, 1, 2050, 129] * 4                    # 20 decodes: the write stays on the current stream
    page, W, B = 16, w.layout["row_width"], 20
    bt, nb, _ = synth.block_tables(seqs, page, extra_blocks=2)
    kv = torch.zeros(nb, 1, page, W, dtype=torch.bfloat16)
    synth.fill_cache(kv[:, 0], w.layout, bt, seqs, seed=3, poison=False)
    g = torch.Generator().manual_seed(12)
    c = (torch.randn(B, W, generator=g) * synth.latent_columns(w.layout)).to(torch.bfloat16).to(dev)
    pos = torch.tensor(seqs) - 1
    slots = (bt[torch.arange(B), pos // page].long() * page + pos % page).to(dev)
    q = synth.make_queries(B, seed=13).to(dev)
    builder = LatentAttentionMetadataBuilder(LatentKVSpec(block_size=page, head_size=W), ["l0"], device=dev,
                                             max_num_batched_tokens=64)
    cm = CommonAttentionMetadata(query_start_loc=torch.arange(B + 1, dtype=torch.int32, device=dev),
                                 query_start_loc_cpu=torch.arange(B + 1, dtype=torch.int32),
                                 seq_lens=torch.tensor(seqs, dtype=torch.int32, device=dev),
                                 block_table_tensor=bt.to(dev), slot_mapping=slots, num_reqs=B, num_actual_tokens=B,
                                 max_query_len=1)
    md = builder.build(0, cm)
    impl = LatentAttentionImpl(24, 256, 256 ** -0.5, 4)

    class Layer:
        def __init__(self, latent):
            self.latent = latent
    layer = Layer(lat)
    kv_e, kv_c = kv.to(dev), kv.to(dev)
    out_e = torch.empty(B, 24, 256, dtype=torch.bfloat16, device=dev)
    out_c = torch.empty_like(out_e)
    impl.forward(layer, q, c, pos.to(dev), kv_e, md, out_e)
    compiled = torch.compile(impl.forward, fullgraph=True)
    compiled(layer, q, c, pos.to(dev), kv_c, md, out_c)
    torch.cuda.synchronize()
    dec.check_device_errors(dev)
    assert torch.equal(kv_e, kv_c)
    assert torch.equal(out_e.view(torch.int16), out_c.view(torch.int16))
    ref = oracle.derive(w.k_up, w.v_up, w.k_norm_weight, w.layout, synth.cos_sin_table(4096))
    exp = oracle.decode_fp32(q.cpu(), kv_e[:, 0].cpu(), bt, torch.tensor(seqs), ref, 256 ** -0.5)
    err = (out_c.float().cpu() - exp).abs()
    assert float(err.max()) < 2e-2 and float(err.mean()) < 2e-3
