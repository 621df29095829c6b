"""Weight hand-over across ranks (host logic, world_size 2 over gloo on the CPU):
packing keeps names/shapes/Parameter objects, one broadcast moves every tensor."""
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from rl_quant_b200.glad_model import build_glad
from rl_quant_b200.weight_sync import PackedWeights


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _worker(rank, world, port, q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        torch.manual_seed(100 + rank)
        m = build_glad(seed=rank)                 # ranks start from different weights
        names = {k: (v.shape, v.dtype) for k, v in m.state_dict().items()}
        params_before = {n: p for n, p in m.named_parameters()}
        packed = PackedWeights(m)
        assert {k: (v.shape, v.dtype) for k, v in m.state_dict().items()} == names
        assert all(params_before[n] is p for n, p in m.named_parameters())
        if rank == 0:
            with torch.no_grad():
                for p in m.parameters():
                    p.add_(1e-3 * torch.randn_like(p))
        packed.broadcast(src=0)
        sums = torch.tensor([float(sum(p.double().sum() for p in m.parameters())), float(packed.checksum())],
                            dtype=torch.float64)
        gathered = [torch.zeros_like(sums) for _ in range(world)]
        dist.all_gather(gathered, sums)
        q.put((rank, [g.tolist() for g in gathered]))
    finally:
        dist.destroy_process_group()


def test_packed_broadcast_gloo_two_ranks():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=180)
    for p in procs:
        if p.is_alive():
            p.kill()
    assert all(p.exitcode == 0 for p in procs)
    results = dict(q.get(timeout=5) for _ in range(2))
    for r in (0, 1):
        g = results[r]
        assert g[0] == g[1]                       # identical parameters and bytes on both ranks


def test_packing_single_process_keeps_values():
    m = build_glad(seed=0)
    before = {k: v.clone() for k, v in m.state_dict().items()}
    packed = PackedWeights(m)
    after = m.state_dict()
    for k in before:
        assert torch.equal(before[k], after[k]), k
    assert packed.nbytes >= sum(v.numel() * v.element_size() for k, v in before.items()
                                if not k.endswith("num_batches_tracked"))
    y = m.act_inference(torch.randn(2, 2175))[0]   # the module still runs on the packed storage
    assert y.shape == (2, 29)


def test_pack_layout_matches_the_c_abi():
    """The blob layout the Python packer uses is the one glad_pack_layout computes."""
    from rl_quant_b200 import _native as N
    from rl_quant_b200.weight_sync import pack_layout

    sizes = [1, 255, 256, 257, 0, 4096, 3, 512 * 224]
    items = (N.GladPackItem * len(sizes))(*[N.GladPackItem(None, n, 7) for n in sizes])
    total = N.load().glad_pack_layout(items, len(sizes))
    offs, tot = pack_layout(sizes)
    assert [it.offset for it in items] == offs and total == tot
    assert all(o % 256 == 0 for o in offs)
    # a rejected item: off the layout (the tensor addresses are never dereferenced here)
    for it in items:
        it.tensor = 0x1000
    items[1].offset = 100
    rc = N.load().glad_pack_weights(items, len(sizes), None, total, None)
    assert rc == N.GLAD_ERR_INVALID_ARG and b"256-byte layout" in N.load().glad_last_error()
