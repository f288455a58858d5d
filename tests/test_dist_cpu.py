"""Multi-rank host logic on CPU (gloo, world size 2): tensor-parallel sharding of the decode
layer (column-parallel QKV by head groups, row-parallel O + all-reduce) and expert-parallel
slicing of the MoE bank reproduce the single-rank oracle.  The math is the CPU oracle; what is
under test is okc_b200.layer.shard_weights and the partition of heads / experts / caches."""

import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _tp_worker(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from oracle import attention as oatt
        from oracle import layer as olayer
        from oracle.projection import gemm, rmsnorm
        from okc_b200 import synth
        from okc_b200.layer import LayerConfig, shard_weights
        c = synth.layer_case(B=3, H=256, Hq=8, Hkv=4, D=64, ctx=(10, 90), page=16, pool_pages=40, theta=1e4,
                             device="cpu", seed=7)
        cfg = LayerConfig(hidden=256, num_q_heads=8, num_kv_heads=4, head_dim=64, rope_theta=1e4)
        wqkv_l, wo_l = shard_weights(c["wqkv"], c["wo"], cfg, rank, world)
        lkv, lq = 4 // world, 8 // world
        hs = slice(rank * lkv, (rank + 1) * lkv)
        kc = c["k_cache"][:, :, hs].contiguous()
        vc = c["v_cache"][:, :, hs].contiguous()
        xn = rmsnorm(c["x"], c["norm_w"], 1e-6)
        qkv = gemm(xn, wqkv_l)
        qr, _ = oatt.kv_append(qkv, c["positions"], c["page_table"], kc, vc, c["k_scale"][hs], c["v_scale"][hs],
                               lq, lkv, 64, 1e4)
        o = oatt.attend(qr.to(torch.bfloat16), kc, vc, c["page_table"], c["positions"] + 1, c["k_scale"][hs],
                        c["v_scale"][hs], 64 ** -0.5).to(torch.bfloat16)
        part = gemm(o.reshape(3, lq * 64), wo_l, out_fp32=True)
        dist.all_reduce(part)
        out = (c["x"].float() + part).to(torch.bfloat16)
        if rank == 0:
            full, _ = olayer.decode_layer(c["x"], c["norm_w"], c["wqkv"], c["wo"], c["positions"], c["page_table"],
                                          c["k_cache"].clone(), c["v_cache"].clone(), c["k_scale"], c["v_scale"],
                                          8, 4, 64, 1e4, 1e-6, 64 ** -0.5)
            q.put(float((out.float() - full.float()).abs().max()))
    finally:
        dist.destroy_process_group()


def _ep_worker(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from oracle import moe as omoe
        from okc_b200 import synth
        m = synth.moe_case(T=4, E=8, H=256, I=128, topk=4, device="cpu", seed=3)
        ids, w, _ = omoe.route(m["x"], m["router"], 4)
        per = 8 // world
        sl = slice(rank * per, (rank + 1) * per)
        part = omoe.experts(m["x"], ids, w, m["w13"][sl], m["w13_sf"][sl], m["w13_gs"][sl], m["w2"][sl],
                            m["w2_sf"][sl], m["w2_gs"][sl], expert_lo=rank * per).float()
        dist.all_reduce(part)  # the expert-parallel combine: sum of the ranks' weighted outputs
        if rank == 0:
            full = omoe.experts(m["x"], ids, w, m["w13"], m["w13_sf"], m["w13_gs"], m["w2"], m["w2_sf"],
                                m["w2_gs"]).float()
            q.put(float((part - full).abs().max() / full.abs().max()))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("worker", [_tp_worker, _ep_worker])
def test_two_rank_partition_matches_single_rank(worker):
    ctx = mp.get_context("spawn")
    q = ctx.SimpleQueue()
    port = _free_port()
    procs = [ctx.Process(target=worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=240)
        assert p.exitcode == 0
    err = q.get()
    assert err < 2e-2, err


def test_shard_weights_rejects_indivisible_heads():
    from okc_b200.layer import LayerConfig, shard_weights
    cfg = LayerConfig(hidden=64, num_q_heads=6, num_kv_heads=3, head_dim=8)
    w = torch.zeros(((6 + 6) * 8, 64))
    with pytest.raises(ValueError):
        shard_weights(w, torch.zeros((64, 48)), cfg, 0, 2)
