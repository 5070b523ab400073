"""Layer sharding on CPU: partitions, Philox offsets across ranks, and the collectives of
the sharded step under gloo with world_size 2, including a rank that dies before the
Kalman all-reduce (detected on the host, no GPU involved)."""
import ctypes
import datetime
import os
import socket
import sys

import pytest
import torch
import torch.multiprocessing as mp

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _paths():
    for p in (ROOT, os.path.join(ROOT, "ds-mezo_b200"), os.path.join(ROOT, "tests")):
        if p not in sys.path:
            sys.path.insert(0, p)


_paths()


@pytest.fixture(scope="module")
def L():
    from dsmezo_b200 import build
    build.build()
    from dsmezo_b200 import _lib
    return _lib.lib()


@pytest.mark.parametrize("layers,world", [(28, 1), (28, 2), (28, 8), (80, 8), (4, 3), (3, 4)])
def test_partition_is_contiguous_and_balanced(layers, world):
    from dsmezo_b200 import partition_layers
    parts = partition_layers(layers, world)
    assert len(parts) == world
    assert parts[0].start == 0 and parts[-1].stop == layers
    for a, b in zip(parts, parts[1:]):
        assert a.stop == b.start
    sizes = [len(p) for p in parts]
    assert max(sizes) - min(sizes) <= 1


def test_partition_by_weight():
    from dsmezo_b200 import partition_layers
    parts = partition_layers(6, 2, [1, 1, 1, 1, 1, 10])
    assert [len(p) for p in parts] == [5, 1]


def _plan_increment(L, mods, bases, rank_r, offsets):
    """rng increment of a host-only plan over `mods` (basis indices into `bases`) whose draws
    sit at the given per-module offsets."""
    from dsmezo_b200 import _lib
    specs = (_lib.ModuleSpec * len(mods))()
    for i, m in enumerate(mods):
        s = specs[i]
        for f in ("A", "B", "pos_A", "pos_B", "neg_A", "neg_B", "mu_A", "mu_B", "var_A", "var_B", "z_A", "z_B"):
            setattr(s, f, 0x10000)
        s.d_out, s.d_in, s.r, s.ld_A, s.ld_B = m.d_out, m.d_in, rank_r, rank_r, m.d_in
        s.basis, s.layer = m.basis, m.layer
    bs = (_lib.BasisSpec * len(bases))()
    for i, b in enumerate(bases):
        bs[i].H, bs[i].h_dtype, bs[i].T, bs[i].D, bs[i].ld_H, bs[i].V, bs[i].R = 0x10000, 1, b.T, b.D, b.D, 0x10000, rank_r
    d = _lib.PlanDesc()
    d.copy_dtype, d.num_modules, d.modules, d.num_bases, d.bases = 1, len(mods), specs, len(bases), bs
    d.sm_count, d.max_threads_per_sm = 148, 2048
    arr = (ctypes.c_uint64 * len(mods))(*offsets)
    d.module_rng_offsets = arr
    h = ctypes.c_void_p()
    assert L.dsmz_plan_create(ctypes.byref(d), ctypes.byref(h)) == 0
    inc = L.dsmz_plan_rng_increment(h)
    L.dsmz_plan_destroy(h)
    return inc


@pytest.mark.parametrize("layers,world", [(8, 2), (8, 3), (28, 8), (3, 2)])
def test_units_cover_the_model_once_and_offsets_follow_controller_order(L, layers, world):
    """Every module lands on exactly one rank, ranks hold contiguous runs of units, and each
    module's draws sit at its place in the whole model's controller order, so the sharded
    step draws the same Gaussians as one GPU (the reference's per-module torch.randn order)."""
    from dsmezo_b200 import draw_increments, shard_layout, transformer_adapter_shapes
    rank_r = 64
    lay = shard_layout(layers, 3584, 18944, 512, rank_r, 4096, world, 148, 2048)
    mods, bases = transformer_adapter_shapes(layers, 3584, 18944, 512, 4096)
    assert lay.ranges[0].start == 0 and lay.ranges[-1].stop == 4 * layers
    for a, b in zip(lay.ranges, lay.ranges[1:]):
        assert a.stop == b.start
    seen = [(m.layer, m.name) for rm in lay.rank_modules for m in rm]
    assert sorted(seen) == sorted((m.layer, m.name) for m in mods) and len(set(seen)) == len(seen)
    incs = draw_increments(mods, rank_r, rank_r, 148, 2048)
    prefix = 0
    for m, inc in zip(mods, incs):
        assert lay.offsets[(m.layer, m.name)] == prefix
        prefix += inc
    total = 0
    for r in range(world):
        rm, rb = lay.rank_modules[r], lay.rank_bases[r]
        for m in rm:                       # each module's basis is its unit's
            assert rb[m.basis].layer == m.layer and rb[m.basis].name == {
                "q_proj": "qkv", "k_proj": "qkv", "v_proj": "qkv", "o_proj": "o", "gate_proj": "gate_up",
                "up_proj": "gate_up", "down_proj": "down"}[m.name]
        if rm:
            total += _plan_increment(L, rm, rb, rank_r, lay.module_offsets(r))
    assert total == prefix == lay.rng_increment_total


@pytest.mark.parametrize("world,bound", [(8, 1.08), (4, 1.05), (2, 1.03)])
def test_unit_partition_balances_the_7b_set(world, bound):
    # whole layers on 8 ranks give 4 layers against a mean of 3.5 (1.14); units do better
    from dsmezo_b200.sharding import model_units, partition_layers, unit_weight
    units = model_units(28)
    w = [unit_weight(u, 3584, 18944, 512, 64, 4096) for u in units]
    parts = partition_layers(len(units), world, w)
    loads = [sum(w[i] for i in p) for p in parts]
    assert max(loads) / (sum(loads) / world) <= bound


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, mode, q):
    _paths()
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=8))
    try:
        from dsmezo_b200.sharding import allreduce_sums, broadcast_scalar, gather_arena
        if mode == "ok":
            sums = torch.tensor([1.5 * (rank + 1), 2.0 ** rank], dtype=torch.float64)
            allreduce_sums(sums)
            dd = broadcast_scalar(3.25 if rank == 0 else -1.0)
            cap = 6
            local = torch.full((cap,), float(rank + 1))
            local[4 + rank:] = 0.0                      # ranks of unequal size, padded
            out = torch.empty(cap * world)
            gather_arena(out, local)
            q.put((rank, "ok", sums.tolist(), dd, out.tolist()))
        elif mode in ("stall", "exit_between"):
            import time
            from dsmezo_b200.sharding import Collectives, CollectiveTimeout
            coll = Collectives(timeout_s=1.5)
            sums = torch.ones(2, dtype=torch.float64)
            coll.all_reduce(sums, "step 1 all-reduce")
            coll.settle()                                # step 1 completes on both ranks
            if rank == 1:
                if mode == "exit_between":
                    os._exit(3)                          # leaves between steps, nothing in flight
                time.sleep(6.0)                          # stalls past rank 0's limit
                os._exit(0)
            t0 = time.monotonic()
            try:
                coll.all_reduce(sums, "step 2 all-reduce")
                coll.settle()
                q.put((rank, "no error", None, None, None))
            except CollectiveTimeout as e:
                q.put((rank, "timeout", time.monotonic() - t0, None, None))
            except Exception as e:                      # peer gone: the collective fails
                q.put((rank, "detected", type(e).__name__, time.monotonic() - t0, None))
        else:
            if rank == 1:
                os._exit(3)                              # dies before the all-reduce
            sums = torch.ones(2, dtype=torch.float64)
            try:
                allreduce_sums(sums)
                q.put((rank, "no error", None, None, None))
            except Exception as e:                      # peer gone: the collective fails
                q.put((rank, "detected", type(e).__name__, None, None))
    finally:
        try:
            dist.destroy_process_group()
        except Exception:
            pass


def _run(mode, world=2):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, mode, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = []
    for _ in range(world if mode == "ok" else 1):
        results.append(q.get(timeout=60))
    for p in procs:
        p.join(timeout=30)
        if p.is_alive():
            p.kill()
    return sorted(results)


def test_collectives_of_the_sharded_step_gloo():
    res = _run("ok")
    for rank, status, sums, dd, out in res:
        assert status == "ok"
        assert sums == [1.5 + 3.0, 1.0 + 2.0]
        assert dd == 3.25
        assert out == [1.0] * 4 + [0.0] * 2 + [2.0] * 5 + [0.0]


def test_rank_failure_is_detected_on_the_host():
    res = _run("fail")
    assert res[0][0] == 0 and res[0][1] == "detected"


def test_stalled_peer_ends_in_a_bounded_timeout():
    # rank 1 stalls past the 1.5 s limit: rank 0's bounded wait ends with CollectiveTimeout
    # well before the process group's own 8 s timeout
    res = _run("stall")
    rank, status, waited = res[0][:3]
    assert rank == 0 and status == "timeout" and 1.4 <= waited < 6.0


def test_peer_that_leaves_between_steps_is_detected():
    # rank 1 exits after step 1 with nothing in flight: rank 0's next collective fails or
    # runs out of its 1.5 s limit instead of hanging
    res = _run("exit_between")
    rank, status = res[0][:2]
    assert rank == 0 and status in ("timeout", "detected")


@pytest.mark.parametrize("world,K", [(1, 1), (2, 1), (3, 2)])
def test_export_index_finds_every_adapter_in_the_gathered_buffer(world, K):
    # every rank's local arena (K directions, `cap` apart) filled with a code per (rank,
    # direction, module, factor), gathered rank-major as the all-gather lays it out
    from dsmezo_b200.sharding import export_index, partition_layers, peft_prefix
    from dsmezo_b200 import transformer_adapter_shapes
    layers, hidden, inter, kv, r, tokens = 5, 64, 160, 16, 4, 8
    ranges = partition_layers(layers, world)
    rank_mods = [transformer_adapter_shapes(layers, hidden, inter, kv, tokens, layer_range=lr)[0] for lr in ranges]
    sizes = [sum(m.d_out * r + r * m.d_in for m in ms) for ms in rank_mods]
    cap = max(sizes) + 3                                  # padded shards
    locals_ = []
    for rk, ms in enumerate(rank_mods):
        arena = torch.full((K * cap,), -1.0)
        for k in range(K):
            n = k * cap
            for i, m in enumerate(ms):
                arena[n:n + m.d_out * r] = 1000 * rk + 100 * k + 2 * i
                n += m.d_out * r
                arena[n:n + r * m.d_in] = 1000 * rk + 100 * k + 2 * i + 1
                n += r * m.d_in
        locals_.append(arena)
    gathered = torch.cat(locals_)
    for k in range(K):
        idx = export_index(rank_mods, r, K * cap, k * cap)
        assert len(idx) == 2 * 7 * layers
        for rk, ms in enumerate(rank_mods):
            for i, m in enumerate(ms):
                pre = peft_prefix(m.layer, m.name)
                oA, shA = idx[f"{pre}.lora_B.weight"]             # the factor A (d_out x r)
                oB, shB = idx[f"{pre}.lora_A.weight"]             # the factor B (r x d_in)
                assert shA == (m.d_out, r) and shB == (r, m.d_in)
                assert torch.all(gathered[oA:oA + m.d_out * r] == 1000 * rk + 100 * k + 2 * i)
                assert torch.all(gathered[oB:oB + r * m.d_in] == 1000 * rk + 100 * k + 2 * i + 1)
    assert "base_model.model.model.layers.0.self_attn.q_proj.lora_A.weight" in export_index(rank_mods, r, cap)
    assert "base_model.model.model.layers.4.mlp.down_proj.lora_B.weight" in export_index(rank_mods, r, cap)
