"""Worker for test_gpu_multi.py (launched by torch.distributed.run, one rank per GPU).

Calibrates every rank's bases against a one-GPU calibration, then runs two layer-sharded
steps and, on rank 0, the same steps on one GPU; compares every rank's gathered factors, pos
and neg of the last step, and their PEFT-named exports, with the single-GPU ones. The
factor gather mode comes from DSMZ_FACTOR_GATHER (copy-engine, fused or nccl), the
perturbation kernel from DSMZ_PERTURB (tensor-cores or cuda-cores). Prints MULTI_OK."""
import datetime
import os
import sys

import torch
import torch.distributed as dist

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, os.path.join(ROOT, "ds-mezo_b200"))

CFG = dict(layers=3, hidden=512, inter=1536, kv=128, rank_r=16, tokens=256)   # 12 units: ranks split a layer
EPS, TOTAL = 1e-3, 100
DDS = (4.5, -2.0)                       # the steps' projected-gradient scalars


def init_units(step):
    """Seeded state per module and per basis, so the union of the shards (which may split a
    layer) equals the one-GPU set."""
    from dsmezo_b200.adapter_set import INPUT_ORDER, MODULE_NAMES
    a = step.aset
    for i, m in enumerate(a.modules):
        g = torch.Generator(device=a.device)
        g.manual_seed(1000 + 16 * m.layer + MODULE_NAMES.index(m.name))
        a.A(i).copy_(torch.randn(a.A(i).shape, generator=g, device=a.device))
        a.B(i).copy_(torch.randn(a.B(i).shape, generator=g, device=a.device))
        a.A(i, a.mu).copy_(torch.randn(a.A(i).shape, generator=g, device=a.device))
        a.B(i, a.mu).copy_(torch.randn(a.B(i).shape, generator=g, device=a.device))
    for b, s in enumerate(a.bases):
        g = torch.Generator(device=a.device)
        g.manual_seed(5000 + 16 * s.layer + INPUT_ORDER.index(s.name))
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
    mode = os.environ.get("DSMZ_FACTOR_GATHER", "copy-engine")
    tcp = os.environ.get("DSMZ_PERTURB", "tensor-cores") == "tensor-cores"
    st = ShardedStep(**CFG, eps=EPS, total_steps=TOTAL, generator=gen, device=dev, process_group=dist.group.WORLD,
                     factor_gather=mode, tensor_core_perturb=tcp, fused_gather=True)
    assert st.aset.perturb_uses_tensor_cores == tcp
    init_units(st)
    # first-step calibration: each rank's bases equal the one-GPU calibration's, and every
    # rank's generator ends where the one-GPU calibration leaves it
    cgen = torch.Generator(device=dev)
    cgen.manual_seed(11)
    st.calibrate(generator=cgen)
    ref1 = ShardedStep(**CFG, eps=EPS, total_steps=TOTAL, generator=torch.Generator(device=dev), device=dev,
                       process_group=None)
    init_units(ref1)
    cg1 = torch.Generator(device=dev)
    cg1.manual_seed(11)
    ref1.calibrate(generator=cg1)
    torch.cuda.synchronize()
    assert cgen.get_offset() == cg1.get_offset(), "calibration advanced the generators differently"
    want_v = {(s.layer, s.name): ref1.aset.V(b) for b, s in enumerate(ref1.aset.bases)}
    for b, s in enumerate(st.aset.bases):
        err = float((st.aset.V(b) - want_v[(s.layer, s.name)]).abs().max())
        assert err < 1e-6, ("calibrated basis", s.layer, s.name, err)
    # the one-GPU step below starts from the same calibrated bases
    calibrated = {k: v.clone() for k, v in want_v.items()}
    del ref1
    for dd in DDS:                           # the second step's copies follow the first's
        st.perturb()
        pn = st.gather("pos", "neg")
        pn = {k: v.clone() for k, v in pn.items()}
        st.update(st.broadcast_dd(dd))
        st.gather("factors")
    st.synchronize()                         # the factors gather overlaps what follows it
    fac = st.gathered["factors"].clone()
    assert st.aset.device_error() == 0
    if rank == 0:
        g1 = torch.Generator(device=dev)
        g1.manual_seed(7)
        one = ShardedStep(**CFG, eps=EPS, total_steps=TOTAL, generator=g1, device=dev, process_group=None,
                          tensor_core_perturb=tcp)
        init_units(one)
        for b, s in enumerate(one.aset.bases):
            one.aset.V(b).copy_(calibrated[(s.layer, s.name)])
        for dd in DDS:
            one.perturb()
            one.update(dd)
        torch.cuda.synchronize()
        assert g1.get_offset() == gen.get_offset(), "generators advanced differently"
        # every adapter, keyed as the reference's PEFT file, from the gathered buffers equals
        # the one-GPU set's (ranks may split a layer, so compare by name, not by position)
        for which, full in (("factors", fac), ("pos", pn["pos"]), ("neg", pn["neg"])):
            st.gathered[which].copy_(full)
            got, want = st.export_adapters(which), one.export_adapters(which)
            assert got.keys() == want.keys() and len(got) == 2 * 7 * CFG["layers"]
            for k in want:
                assert got[k].shape == want[k].shape and got[k].dtype == torch.bfloat16, k
                err = float((got[k].float() - want[k].float()).abs().max() / want[k].float().abs().max())
                assert err < 1e-5, (which, k, err)
        print("MULTI_OK", flush=True)
    # every rank's +/- copies reached every rank through the perturbation's peer stores when
    # the fused gather is on (NVLink); the comparison above covers either path
    if rank == 0:
        print("FUSED_GATHER", st.fused_gather, st.factor_gather, flush=True)
    dist.barrier(device_ids=[local])
    st.close()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
