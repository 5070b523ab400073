"""Worker for test_gpu_multi.py (launched by torch.distributed.run, one rank per GPU).

Runs one layer-sharded step and, on rank 0, the same step on one GPU; compares every
rank's gathered factors, pos and neg, and their PEFT-named exports, with the single-GPU
ones. Prints MULTI_OK."""
import datetime
import os
import sys

import torch
import torch.distributed as dist

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, os.path.join(ROOT, "ds-mezo_b200"))

CFG = dict(layers=4, hidden=512, inter=1536, kv=128, rank_r=16, tokens=256)
EPS, TOTAL = 1e-3, 100


def init_by_layer(step, layers):
    """Per-layer seeded state, so the union of the shards equals the one-GPU set."""
    a = step.aset
    per = 7
    for li_local, li in enumerate(layers):
        g = torch.Generator(device=a.device)
        g.manual_seed(1000 + li)
        for j in range(per):
            i = li_local * per + j
            a.A(i).copy_(torch.randn(a.A(i).shape, generator=g, device=a.device))
            a.B(i).copy_(torch.randn(a.B(i).shape, generator=g, device=a.device))
            a.A(i, a.mu).copy_(torch.randn(a.A(i).shape, generator=g, device=a.device))
            a.B(i, a.mu).copy_(torch.randn(a.B(i).shape, generator=g, device=a.device))
        for k in range(4):
            b = li_local * 4 + k
            s = a.bases[b]
            a.V(b).copy_(torch.linalg.qr(torch.randn(s.D, CFG["rank_r"], generator=g, device=a.device))[0])
            a.H(b).copy_(torch.randn(s.T, s.D, generator=g, device=a.device) * torch.exp(
                torch.randn(s.D, generator=g, device=a.device)))
    a.var.fill_(EPS ** 2)
    a.sync_shadow()


def main():
    from dsmezo_b200 import ShardedStep
    local = int(os.environ["LOCAL_RANK"])
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=60), device_id=dev)
    rank, world = dist.get_rank(), dist.get_world_size()
    gen = torch.Generator(device=dev)
    gen.manual_seed(7)
    st = ShardedStep(**CFG, eps=EPS, total_steps=TOTAL, generator=gen, device=dev, process_group=dist.group.WORLD)
    init_by_layer(st, st.layout.ranges[rank])
    st.perturb()
    pn = st.gather("pos", "neg")
    pn = {k: v.clone() for k, v in pn.items()}
    st.update(st.broadcast_dd(4.5))
    fac = st.gather("factors")["factors"].clone()
    assert st.aset.device_error() == 0
    if rank == 0:
        g1 = torch.Generator(device=dev)
        g1.manual_seed(7)
        one = ShardedStep(**CFG, eps=EPS, total_steps=TOTAL, generator=g1, device=dev, process_group=None)
        init_by_layer(one, range(CFG["layers"]))
        one.perturb()
        one.update(4.5)
        torch.cuda.synchronize()
        assert g1.get_offset() == gen.get_offset(), "generators advanced differently"
        off = 0
        for r in range(world):
            n = st.layout.sizes[r]
            for name, full in (("factors", fac), ("pos", pn["pos"]), ("neg", pn["neg"])):
                got = st.full_view(full, r).float()
                arena = one.aset.export_factors if name == "factors" else getattr(one.aset, name)
                want = arena[off:off + n].float()
                err = float((got - want).abs().max() / want.abs().max())
                assert err < 1e-5, (r, name, err)
            off += n
        # the PEFT export from the gathered buffers names and places every adapter as the
        # one-GPU set's export does
        for which in ("factors", "pos"):
            got, want = st.export_adapters(which), one.export_adapters(which)
            assert got.keys() == want.keys() and len(got) == 2 * 7 * CFG["layers"]
            for k in want:
                assert got[k].shape == want[k].shape and got[k].dtype == torch.bfloat16, k
                err = float((got[k].float() - want[k].float()).abs().max() / want[k].float().abs().max())
                assert err < 1e-5, (which, k, err)
        print("MULTI_OK", flush=True)
    dist.barrier(device_ids=[local])
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
