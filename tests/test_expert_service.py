"""SWARMEX1 packets, codecs, expert worker service with microshards (CPU)."""
import asyncio

import pytest
import torch

from swarm_inference_lab_b200.runtime.expert_service import (ExpertClient, ExpertService, ExpertStore, Microshard,
                                                             reduce_fixed_order, split_microshards)
from swarm_inference_lab_b200.transport.expert_wire import (ExpertPacket, ExpertWireError, decode_packet,
                                                            decode_tensor, encode_packet, encode_tensor)


def test_packet_roundtrip_and_codecs():
    p = ExpertPacket({"kind": "x"})
    t = torch.randn(5, 64)
    for codec in ("raw_fp32", "raw_fp16", "raw_bf16", "int8_per_vector"):
        encode_tensor(p, codec, t, codec)
    q = decode_packet(encode_packet(p))
    assert torch.equal(decode_tensor(q, "raw_fp32"), t)
    assert (decode_tensor(q, "raw_fp16") - t).abs().max() < 1e-2
    assert (decode_tensor(q, "raw_bf16") - t).abs().max() < 3e-2
    assert ((decode_tensor(q, "int8_per_vector") - t).abs().max(dim=1).values
            <= t.abs().max(dim=1).values / 127 * 0.51 + 1e-6).all()
    raw = encode_packet(p)
    with pytest.raises(ExpertWireError):
        decode_packet(raw[:-1])
    with pytest.raises(ExpertWireError):
        decode_packet(b"NOTMAGIC" + raw[8:])


def test_expert_service_whole_and_microshards():
    H, I, E = 32, 48, 4
    g = torch.Generator().manual_seed(0)
    W = {e: (torch.randn(I, H, generator=g) * 0.1, torch.randn(I, H, generator=g) * 0.1,
             torch.randn(H, I, generator=g) * 0.1) for e in range(E)}
    x = torch.randn(6, H, generator=g)
    ids = torch.tensor([[0, 1], [2, 3], [1, 2], [0, 3], [3, 1], [2, 0]])
    wts = torch.rand(6, 2, generator=g)

    def expert(e, rows):
        gt, up, dn = W[e]
        return (torch.nn.functional.silu(rows @ gt.T) * (rows @ up.T)) @ dn.T
    ref = torch.stack([sum(wts[r, s] * expert(int(ids[r, s]), x[r:r + 1])[0] for s in range(2))
                       for r in range(6)])

    async def main():
        whole = ExpertStore()
        for e in range(E):
            whole.add(Microshard(0, e, 0, I), *W[e])
        svc = ExpertService(whole, max_inflight=2)
        port = await svc.start()
        svc.accept_lease("lease-1")
        cli = ExpertClient("127.0.0.1", port)
        rep = await cli.run(request_id="r1", layer=0, rows=x, expert_ids=ids, weights=wts, lease_hash="lease-1")
        assert rep.header["status"] == "OK"
        assert torch.allclose(decode_tensor(rep, "weighted_sum"), ref, atol=1e-5)
        await cli.run(request_id="r1", layer=0, rows=x, expert_ids=ids, weights=wts, lease_hash="lease-1")
        assert svc.stats["cache_hits"] == 1
        bad = await cli.run(request_id="r2", layer=0, rows=x, expert_ids=ids, weights=wts, lease_hash="nope")
        assert bad.header["status"] == "ERROR"
        cli.close()
        await svc.close()
        # microshards: three workers each own a slice of every expert
        shards = [ExpertStore() for _ in range(3)]
        svcs = []
        for e in range(E):
            for k, ms in enumerate(split_microshards(0, e, I, 3)):
                shards[k].add(ms, *W[e])
        partials = {}
        for k, st in enumerate(shards):
            s = ExpertService(st)
            p = await s.start()
            s.accept_lease("lease-1")
            c = ExpertClient("127.0.0.1", p)
            r = await c.run(request_id=f"m{k}", layer=0, rows=x, expert_ids=ids, weights=wts,
                            lease_hash="lease-1", mode="per_expert_exact")
            partials[k] = (decode_tensor(r, "outputs") * wts[..., None]).sum(1)
            c.close()
            svcs.append(s)
        for s in svcs:
            await s.close()
        assert torch.allclose(reduce_fixed_order(partials), ref, atol=1e-5)

    asyncio.run(main())
