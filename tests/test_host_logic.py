"""Host-side logic of the GDN path, on CPU: context mirror, head sharding,
layer split, state-pool layout and slot lifecycle, layer construction and
weight loading (no kernels run)."""
import types

import pytest
import torch


def test_context_mirror_fields(pkg):
    Cx = pkg.context
    fields = [f for f in Cx.Context.__dataclass_fields__]
    assert fields == ["cu_seqlens_q", "cu_seqlens_k", "max_seqlen_q", "max_seqlen_k",
                      "slot_mapping", "block_tables", "num_decode_tokens", "flashinfer_decode",
                      "flashinfer_prefill", "draft_slot_mapping", "draft_block_tables",
                      "linear_state_ids", "lens_q", "vision_embeds"]
    ids = torch.tensor([3, 1])
    Cx.set_context(torch.tensor([0, 1, 2]), None, 1, 1, linear_state_ids=ids, lens_q=[1, 1])
    c = Cx.get_context()
    assert c.max_seqlen_q == 1 and c.linear_state_ids is ids and c.lens_q == [1, 1]
    Cx.reset_context()
    assert Cx.get_context().linear_state_ids is None


@pytest.mark.parametrize("G", [1, 2, 4, 8])
def test_head_shard_covers_heads_and_keeps_gqa_local(pkg, G):
    P = pkg.parallel
    HV, HK = 32, 16
    seen_v, seen_k = [], []
    for r in range(G):
        vs, ks = P.head_shard(HV, HK, G, r)
        seen_v += list(range(HV))[vs]
        seen_k += list(range(HK))[ks]
        rep = HV // HK
        for hv in range(HV)[vs]:
            assert hv // rep in range(HK)[ks]          # h_k = h_v // rep stays local
    assert seen_v == list(range(HV)) and seen_k == list(range(HK))


def test_conv_layout_shard_roundtrip(pkg):
    P = pkg.parallel
    kd, vd = 16 * 4, 32 * 4          # 16 k-heads, 32 v-heads of dim 4
    w = torch.arange((2 * kd + vd) * 3, dtype=torch.float32).view(2 * kd + vd, 3)
    for G in (1, 2, 4, 8):
        shards = [P.conv_layout_shard(w, kd, vd, G, r) for r in range(G)]
        qs = torch.cat([s[:kd // G] for s in shards])
        ks = torch.cat([s[kd // G:2 * kd // G] for s in shards])
        vs = torch.cat([s[2 * kd // G:] for s in shards])
        assert torch.equal(torch.cat([qs, ks, vs]), w)


def test_split_layers_and_peers(pkg):
    P = pkg.parallel
    assert [P.split_layers(24, 8, r) for r in range(8)] == [(3 * r, 3 * r + 3) for r in range(8)]
    assert [P.split_layers(24, 5, r) for r in range(5)] == [(0, 5), (5, 10), (10, 15),
                                                             (15, 20), (20, 24)]
    assert P.pp_peers(0, 2, 2) == (None, 2) and P.pp_peers(3, 2, 2) == (1, None)


def test_state_pool_layout_and_lifecycle(pkg):
    SP = pkg.state_pool
    mods = [types.SimpleNamespace(s_cache=None, conv_cache=None, num_v_heads=4, head_k_dim=8,
                                  head_v_dim=8, conv_dim=48, conv_kernel=4) for _ in range(3)]
    pools = SP.StatePools(mods, num_slots=5, device="cpu")
    assert pools.s_pool.shape == (6, 3, 4, 8, 8) and pools.conv_pool.shape == (6, 3, 48, 3)
    assert pools.dummy_slot == 5
    v = mods[1].s_cache
    assert v.shape == (6, 4, 8, 8) and v.stride(0) == 3 * 4 * 8 * 8
    assert v.stride(1) == 64 and v.stride(2) == 8 and v.stride(3) == 1
    assert mods[2].conv_cache.stride(0) == 3 * 48 * 3 and mods[2].conv_cache.stride(1) == 3
    pools.s_pool.fill_(1.0); pools.conv_pool.fill_(1.0)
    pools.reset(torch.tensor([4, 1]))
    assert pools.s_pool[[1, 4]].abs().sum() == 0 and pools.s_pool[[0, 2, 3, 5]].min() == 1
    assert SP.StatePools.bytes_per_slot(18, 32, 128, 128, 8192, 4) == 18 * (2 ** 21 + 49152)


def _cfg(hidden=64, HK=2, HV=4, D=16):
    return types.SimpleNamespace(hidden_size=hidden, linear_num_key_heads=HK,
                                 linear_num_value_heads=HV, linear_key_head_dim=D,
                                 linear_value_head_dim=D, linear_conv_kernel_dim=4,
                                 rms_norm_eps=1e-6)


def test_layer_parameters_match_reference_names_and_shapes(pkg):
    m = pkg.layer.Qwen3_5GatedDeltaNet(_cfg())
    shapes = {n: tuple(p.shape) for n, p in m.named_parameters()}
    assert shapes == {
        "in_proj_qkv.weight": (2 * 32 + 64, 64), "in_proj_z.weight": (64, 64),
        "in_proj_b.weight": (4, 64), "in_proj_a.weight": (4, 64),
        "conv1d.weight": (128, 1, 4), "A_log": (4,), "dt_bias": (4,),
        "norm.weight": (16,), "out_proj.weight": (64, 64)}
    for n in ("num_v_heads", "head_k_dim", "head_v_dim", "conv_dim", "conv_kernel"):
        assert hasattr(m, n)
    assert m.s_cache is None and m.conv_cache is None


def test_layer_fused_projection_aliases_and_loads(pkg):
    m = pkg.layer.Qwen3_5GatedDeltaNet(_cfg())
    Fw = m._fused_weight()
    w = torch.randn(128, 64)
    m.in_proj_qkv.weight.weight_loader(m.in_proj_qkv.weight, w)
    assert torch.equal(Fw[:128], w)
    sd = {k: torch.randn_like(v) for k, v in m.state_dict().items()}
    m.load_state_dict(sd)
    Fw = m._fused_weight()
    assert torch.equal(Fw[128:192], sd["in_proj_z.weight"])
    assert torch.equal(Fw[192:196], sd["in_proj_b.weight"])
    assert torch.equal(Fw[196:200], sd["in_proj_a.weight"])
    m2 = m.to(torch.float64)                           # breaks aliasing; rebuilt once
    Fw2 = m2._fused_weight()
    assert Fw2.dtype == torch.float64 and Fw2[:128].data_ptr() == m2.in_proj_qkv.weight.data_ptr()
    assert torch.equal(Fw2[128:192].float(), sd["in_proj_z.weight"])


def test_layer_tp_sharded_loading(pkg):
    """Rank r of a 2-way group loads its head shard of every parameter."""
    for r in range(2):
        P = types.SimpleNamespace(get_tp_rank=lambda r=r: r, get_tp_size=lambda: 2,
                                  get_tp_group=lambda: None)
        m = pkg.layer.Qwen3_5GatedDeltaNet(_cfg(), parallel=P)
        assert m.num_v_heads == 2 and m.num_k_heads == 1 and m.conv_dim == 64
        full = torch.arange(128 * 64, dtype=torch.float32).view(128, 64)
        m.in_proj_qkv.weight.weight_loader(m.in_proj_qkv.weight, full)
        expect = pkg.parallel.conv_layout_shard(full, 32, 64, 2, r)
        assert torch.equal(m.in_proj_qkv.weight.data, expect)
        zfull = torch.arange(64 * 64, dtype=torch.float32).view(64, 64)
        m.in_proj_z.weight.weight_loader(m.in_proj_z.weight, zfull)
        assert torch.equal(m.in_proj_z.weight.data, zfull[32 * r:32 * (r + 1)])
        ofull = torch.arange(64 * 64, dtype=torch.float32).view(64, 64)
        m.out_proj.weight.weight_loader(m.out_proj.weight, ofull)
        assert torch.equal(m.out_proj.weight.data, ofull[:, 32 * r:32 * (r + 1)])
        assert m._v_head_slice == slice(2 * r, 2 * r + 2)


def test_ops_reject_cpu_tensors(pkg):
    ops = pkg.ops
    with pytest.raises(AssertionError):
        ops.rms_norm_gated(torch.zeros(2, 64, dtype=torch.bfloat16),
                           torch.zeros(2, 64, dtype=torch.bfloat16),
                           torch.ones(64, dtype=torch.bfloat16), 1e-6)


def test_debug_checks_of_slot_ids_and_cu_seqlens(pkg):
    """The optional host-side checks: ids inside the pool and unrepeated
    (the last slot, the engine's dummy slot for graph pad rows, may repeat);
    cu_seqlens from 0, non-decreasing, ending at the row count, no sequence
    longer than max_seqlen.  Off by default."""
    ops = pkg.ops
    assert ops._DEBUG_CHECKS is False
    ops.check_slot_ids(torch.tensor([3, 0, 7, 7, 7]), 8)     # 7 is the dummy slot
    with pytest.raises(IndexError):
        ops.check_slot_ids(torch.tensor([0, 8]), 8)
    with pytest.raises(IndexError):
        ops.check_slot_ids([-1], 8)
    with pytest.raises(ValueError, match="appears 2 times"):
        ops.check_slot_ids(torch.tensor([2, 5, 2]), 8)
    ops.check_cu_seqlens(torch.tensor([0, 3, 3, 10], dtype=torch.int32), 10, max_seqlen=7)
    for cu, n, msl in (([1, 3, 10], 10, None), ([0, 5, 4, 10], 10, None), ([0, 3, 9], 10, None),
                       ([0, 3, 10], 10, 6), ([], 0, None)):
        with pytest.raises(ValueError):
            ops.check_cu_seqlens(torch.tensor(cu, dtype=torch.int32), n, max_seqlen=msl)
    try:
        ops.set_debug_checks(True)
        assert ops._DEBUG_CHECKS is True
    finally:
        ops.set_debug_checks(False)
