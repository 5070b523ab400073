"""Sharded optimizer step over one process per GPU.

The step shards by unit: a unit is one module input of one layer (the qkv, o, gate_up or
down activation) with its power-iteration basis and the modules that read it (q, k, v;
o; gate, up; down). Ranks take contiguous runs of units, balanced by their measured cost,
so a rank may hold part of a layer. Each matrix's work is independent; two things cross
ranks:

* the two Kalman sums (sum z*mu, sum z^2*var) are sums over every adapter of the model
  (ds_mezo/controller.py:262-274), so they are all-reduced between the perturbation and
  update phases;
* the random draws: every rank keeps the same torch generator and places each module's
  draws at that module's place in the whole model's controller order (a prefix sum of the
  per-module generator increments), so a sharded step draws exactly what one GPU would.

After the phases, the rollout needs the full adapter set: pos/neg copies for scoring and
the updated factors for the next rollout, both in the copy dtype it loads (bf16 for the
bf16 configs; the fp32 masters stay on their rank). Each rank's arenas are padded to the
largest shard, so each all-gather is one NCCL call on contiguous buffers.
"""
from __future__ import annotations

import time
from dataclasses import dataclass
from typing import Dict, List, Optional, Sequence, Tuple

import torch

from .adapter_set import (INPUT_OF, INPUT_ORDER, MODULE_NAMES, AdapterSet, BasisShape, ModuleShape, ZOController,
                          device_layout, draw_increments, transformer_adapter_shapes)


def partition_layers(layers: int, world: int, weights: Optional[Sequence[float]] = None) -> List[range]:
    """Contiguous layer ranges, one per rank, balanced by per-layer weight (bytes).

    Equal weights give sizes differing by at most one layer, larger ranges first."""
    if world <= 0:
        raise ValueError("world must be positive")
    if weights is None:
        base, extra = divmod(layers, world)
        out, s = [], 0
        for r in range(world):
            n = base + (1 if r < extra else 0)
            out.append(range(s, s + n))
            s += n
        return out
    w = list(weights)
    if len(w) != layers:
        raise ValueError("one weight per layer")
    total = float(sum(w))
    out, s = [], 0
    for r in range(world):
        if r == world - 1:
            out.append(range(s, layers))
            break
        target = total * (r + 1) / world
        e, acc = s, float(sum(w[:s]))
        while e < layers and acc + w[e] / 2.0 <= target:
            acc += w[e]
            e += 1
        out.append(range(s, e))
        s = e
    return out


# ----------------------------------------------------------------------------- collectives
class CollectiveTimeout(RuntimeError):
    """A collective of the sharded step did not complete within its host-side limit (a peer
    stalled or left); the process group has been aborted."""


def _abort(group) -> None:
    """Aborts the process group from a daemon thread: on NCCL the ranks' pending
    collectives end with an error; a backend whose abort waits for the stalled collective
    (gloo) does not hold up the caller, which raises at once."""
    import threading
    import torch.distributed as dist
    fn = getattr(dist.distributed_c10d, "_abort_process_group", None)
    if fn is None:
        return

    def run():
        try:
            fn(group) if group is not None else fn()
        except Exception:
            pass
    threading.Thread(target=run, name="dsmezo-abort", daemon=True).start()


class Collectives:
    """The step's collectives, issued asynchronously, each with a host-side time limit.

    On NCCL a collective is ordered on the current CUDA stream at once (work.wait() makes
    the stream, not the host, wait), so the step's kernels see its result without a host
    synchronisation; a watchdog thread polls the pending handles, and when one is not
    complete `timeout_s` after it was issued (a peer stalled or left) it aborts the process
    group, so that the collectives of the ranks still waiting end with an error instead of
    hanging, and records a CollectiveTimeout that check() raises at the next phase boundary.
    settle() waits for every pending handle on the host within the same limit (the gloo
    backend, whose handles are host-side, is settled this way)."""

    def __init__(self, group=None, timeout_s: float = 60.0, poll_s: float = 1e-3):
        import threading
        import torch.distributed as dist
        self.group = group
        self.timeout_s = float(timeout_s)
        self.poll_s = float(poll_s)
        self.stream_ordered = dist.get_backend(group) == "nccl"
        self._lock = threading.Lock()
        self._pending: List[Tuple[object, str, float]] = []
        self._error: Optional[BaseException] = None
        self._thread = None
        self._deferred: Dict[str, list] = {}

    # ------------------------------------------------------------------ issue
    def _issue(self, work, what: str, defer: Optional[str] = None) -> None:
        """defer: the current stream does not wait for this collective yet; wait_for(defer)
        orders it later (a collective that overlaps the kernels that follow it)."""
        if self.stream_ordered:
            if defer is None:
                work.wait()                  # the current stream waits for the collective
            else:
                self._deferred.setdefault(defer, []).append(work)
        with self._lock:
            self._pending.append((work, what, time.monotonic() + self.timeout_s))
        if self.stream_ordered and self._thread is None:
            import threading
            self._thread = threading.Thread(target=self._watch, name="dsmezo-collective-watchdog", daemon=True)
            self._thread.start()

    def all_reduce(self, t: torch.Tensor, what: str = "all-reduce") -> None:
        import torch.distributed as dist
        self._issue(dist.all_reduce(t, group=self.group, async_op=True), what)

    def broadcast(self, t: torch.Tensor, src: int, what: str = "broadcast") -> None:
        import torch.distributed as dist
        self._issue(dist.broadcast(t, src=src, group=self.group, async_op=True), what)

    def all_gather_into(self, out: torch.Tensor, local: torch.Tensor, what: str = "all-gather",
                        defer: Optional[str] = None) -> None:
        import torch.distributed as dist
        self._issue(dist.all_gather_into_tensor(out, local, group=self.group, async_op=True), what, defer)

    def wait_for(self, key: str) -> None:
        """Orders the deferred collectives of `key` on the current stream (no host wait)."""
        for work in self._deferred.pop(key, []):
            work.wait()

    # ------------------------------------------------------------------ limits
    def _expire(self, what: str) -> None:
        self._error = CollectiveTimeout(f"{what}: not complete after {self.timeout_s:g} s (a peer stalled or left); "
                                        f"the process group was aborted")
        _abort(self.group)

    def _watch(self) -> None:
        while self._error is None:
            with self._lock:
                items = list(self._pending)
            now = time.monotonic()
            done = set()
            for i, (work, what, deadline) in enumerate(items):
                if work.is_completed():
                    done.add(id(work))
                elif now > deadline:
                    self._expire(what)
                    return
            if done:
                with self._lock:
                    self._pending = [p for p in self._pending if id(p[0]) not in done]
            time.sleep(self.poll_s)

    def check(self) -> None:
        """Raises the recorded failure, if any (non-blocking)."""
        if self._error is not None:
            raise self._error

    def settle(self) -> None:
        """Waits on the host for every pending collective, within each one's limit."""
        self.check()
        for key in list(self._deferred):
            self.wait_for(key)
        with self._lock:
            items = list(self._pending)
        t0 = time.monotonic()
        for work, what, deadline in items:
            while not work.is_completed():
                if self._error is not None:
                    raise self._error
                now = time.monotonic()
                if now > deadline:
                    self._expire(what)
                    raise self._error
                # fine polling while the collective is expected to end soon, coarse after
                time.sleep(2e-5 if now - t0 < 0.01 else self.poll_s)
            work.wait()                      # a failed collective raises here
        with self._lock:
            self._pending = [p for p in self._pending if p[0] not in [w for w, _, _ in items]]


def allreduce_sums(t: torch.Tensor, group=None) -> torch.Tensor:
    """In-place sum of the rank-local Kalman sums over the group."""
    import torch.distributed as dist
    dist.all_reduce(t, group=group)
    return t


def broadcast_scalar(x: float, group=None, src: int = 0, device="cpu") -> float:
    """The scoring rank's scalar (dd) on every rank."""
    import torch.distributed as dist
    t = torch.tensor([float(x)], dtype=torch.float64, device=device)
    dist.broadcast(t, src=src, group=group)
    return float(t.item())


def gather_arena(out: torch.Tensor, local: torch.Tensor, group=None) -> torch.Tensor:
    """All-gather of equal-sized (padded) arenas into `out`, rank-major."""
    import torch.distributed as dist
    dist.all_gather_into_tensor(out, local, group=group)
    return out


# Step cost per activation byte and per adapter element, measured on one B200 at the 7B
# shapes (power iteration 8.02 ms over 6.81 GB of bf16 activations, adapter phase 4.79 ms
# over 161.5 M elements): the weights that balance the ranks.
COST_PER_ACT_BYTE = 8.02e-3 / 6.81e9
COST_PER_ELEMENT = 4.79e-3 / 161.5e6


def model_units(layers: int) -> List[Tuple[int, str]]:
    """Every unit of the model in order: (layer, module input), inputs as INPUT_ORDER."""
    return [(li, g) for li in range(layers) for g in INPUT_ORDER]


def unit_shapes(units: Sequence[Tuple[int, str]], hidden: int, intermediate: int, kv_out: int, tokens: int):
    """Modules (controller order: by layer, then module name) and bases (one per unit, in
    the units' order) of a run of units."""
    dims = {"q_proj": (hidden, hidden), "k_proj": (kv_out, hidden), "v_proj": (kv_out, hidden),
            "o_proj": (hidden, hidden), "gate_proj": (intermediate, hidden), "up_proj": (intermediate, hidden),
            "down_proj": (hidden, intermediate)}
    in_dim = {"qkv": hidden, "o": hidden, "gate_up": hidden, "down": intermediate}
    bases = [BasisShape(li, g, tokens, in_dim[g]) for li, g in units]
    index = {u: i for i, u in enumerate(units)}
    mods = []
    for li in sorted({li for li, _ in units}):
        for name in MODULE_NAMES:
            u = (li, INPUT_OF[name])
            if u in index:
                d_out, d_in = dims[name]
                mods.append(ModuleShape(li, name, d_out, d_in, index[u]))
    return mods, bases


def unit_weight(unit: Tuple[int, str], hidden: int, intermediate: int, kv_out: int, rank_r: int, tokens: int,
                act_bytes: int = 2) -> float:
    mods, bases = unit_shapes([unit], hidden, intermediate, kv_out, tokens)
    elems = sum(m.d_out * rank_r + rank_r * m.d_in for m in mods)
    return COST_PER_ACT_BYTE * bases[0].T * bases[0].D * act_bytes + COST_PER_ELEMENT * elems


@dataclass
class ShardLayout:
    ranges: List[range]            # per rank: its run of units (indices into model_units)
    units: List[Tuple[int, str]]
    rank_modules: List[List[ModuleShape]]
    rank_bases: List[List[BasisShape]]
    increments: List[int]          # per module of the whole model, controller order
    offsets: Dict[Tuple[int, str], int]   # (layer, module name) -> generator offset of its draws
    sizes: List[int]               # factor elements per rank
    capacity: int                  # largest shard

    def module_offsets(self, rank: int) -> List[int]:
        return [self.offsets[(m.layer, m.name)] for m in self.rank_modules[rank]]

    def rng_offset_before(self, rank: int) -> int:
        """Offset of the rank's first module's draws."""
        mods = self.rank_modules[rank]
        return self.offsets[(mods[0].layer, mods[0].name)] if mods else self.rng_increment_total

    @property
    def rng_increment_total(self) -> int:
        return sum(self.increments)


def shard_layout(layers: int, hidden: int, inter: int, kv: int, rank_r: int, tokens: int, world: int,
                 sm_count: int, max_threads_per_sm: int, act_bytes: int = 2) -> ShardLayout:
    units = model_units(layers)
    weights = [unit_weight(u, hidden, inter, kv, rank_r, tokens, act_bytes) for u in units]
    ranges = partition_layers(len(units), world, weights)
    mods, _ = transformer_adapter_shapes(layers, hidden, inter, kv, tokens)
    incs = draw_increments(mods, rank_r, rank_r, sm_count, max_threads_per_sm)
    offsets, off = {}, 0
    for m, inc in zip(mods, incs):
        offsets[(m.layer, m.name)] = off
        off += inc
    rank_modules, rank_bases, sizes = [], [], []
    for r in ranges:
        ms, bs = unit_shapes([units[i] for i in r], hidden, inter, kv, tokens)
        rank_modules.append(ms)
        rank_bases.append(bs)
        sizes.append(sum(m.d_out * rank_r + rank_r * m.d_in for m in ms))
    return ShardLayout(ranges, units, rank_modules, rank_bases, incs, offsets, sizes, max(sizes) if sizes else 0)


# Module path of each adapted projection in a Llama/Qwen decoder, under the PEFT prefix
# the reference builds ("base_model.model." + the module's name, ds_mezo/model_config.py:30-35).
PEFT_PATH = {"q_proj": "self_attn.q_proj", "k_proj": "self_attn.k_proj", "v_proj": "self_attn.v_proj",
             "o_proj": "self_attn.o_proj", "gate_proj": "mlp.gate_proj", "up_proj": "mlp.up_proj",
             "down_proj": "mlp.down_proj"}


def peft_prefix(layer: int, name: str) -> str:
    return f"base_model.model.model.layers.{layer}.{PEFT_PATH[name]}"


def export_index(rank_modules: Sequence[Sequence], rank_r: int, block: int, base: int = 0
                 ) -> Dict[str, Tuple[int, Tuple[int, int]]]:
    """Where each PEFT adapter tensor lies in a buffer that holds every rank's factor arena
    one after another, `block` elements apart, starting at `base` (a direction's offset
    inside a rank's block). Keys follow ds_mezo/backend.py:21-34: lora_A.weight is the
    factor B (r x d_in) and lora_B.weight the factor A (d_out x r), the PiSSA/PEFT swap.
    Values are (element offset, shape). Host only."""
    out = {}
    for rk, mods in enumerate(rank_modules):
        n = rk * block + base
        for m in mods:
            pre = peft_prefix(m.layer, m.name)
            out[f"{pre}.lora_B.weight"] = (n, (m.d_out, rank_r))
            n += m.d_out * rank_r
            out[f"{pre}.lora_A.weight"] = (n, (rank_r, m.d_in))
            n += rank_r * m.d_in
    return out


class ShardedStep:
    """One rank's part of the layer-sharded step (all of it when world == 1)."""

    def __init__(self, layers: int, hidden: int, inter: int, kv: int, rank_r: int, tokens: int, *,
                 eps: float, total_steps: int, generator: torch.Generator, copy_dtype=torch.bfloat16,
                 act_dtype=torch.bfloat16, schedule="cubic", device="cuda", process_group=None, power_iters: int = 3,
                 directions: int = 1, single_pass_power_iter: bool = False, collective_timeout_s: float = 60.0,
                 tensor_core_perturb: bool = True, fused_gather: Optional[bool] = None,
                 factor_gather: Optional[str] = None):
        import torch.distributed as dist
        self.pg = process_group
        self.coll = Collectives(process_group, collective_timeout_s) if process_group is not None else None
        self.world = dist.get_world_size(process_group) if process_group is not None else 1
        self.rank = dist.get_rank(process_group) if process_group is not None else 0
        layout = device_layout(device)
        self.layout = shard_layout(layers, hidden, inter, kv, rank_r, tokens, self.world, *layout)
        self._shape = (layers, hidden, inter, kv, rank_r, tokens)
        mods, bases = self.layout.rank_modules[self.rank], self.layout.rank_bases[self.rank]
        # one direction's draws over the whole model: the stride between directions' draws
        stride = self.layout.rng_increment_total
        cap = self.layout.capacity
        self.gathered = {name: torch.zeros(cap * self.world * (1 if name == "factors" else directions),
                                           dtype=copy_dtype, device=device)
                         for name in ("factors", "pos", "neg")} if self.world > 1 else None
        # on several ranks the +/- copies are written straight into this rank's slice of the
        # gather buffers (an in-place all-gather, or the peers' stores of the fused one)
        sl = slice(self.rank * directions * cap, (self.rank + 1) * directions * cap)
        self.aset = AdapterSet(mods, bases, rank_r, rank_r, copy_dtype=copy_dtype, act_dtype=act_dtype,
                               device=device, module_rng_offsets=self.layout.module_offsets(self.rank),
                               layout=layout, capacity=cap, directions=directions,
                               rng_direction_stride=stride, single_pass_power_iter=single_pass_power_iter,
                               tensor_core_perturb=tensor_core_perturb,
                               pos_buffer=self.gathered["pos"][sl] if self.world > 1 else None,
                               neg_buffer=self.gathered["neg"][sl] if self.world > 1 else None,
                               shadow_buffer=(self.gathered["factors"][self.rank * cap:(self.rank + 1) * cap]
                                              if self.world > 1 and copy_dtype != torch.float32 else None))
        self.ctl = ZOController(self.aset, eps, total_steps, generator, power_iters=power_iters, schedule=schedule,
                                process_group=None, rng_increment_total=stride * directions)
        if factor_gather is None:
            # copy engines beside the next power iteration are measured and tested on two GPUs;
            # with more ranks the update's peer stores (measured at four and eight) stand
            factor_gather = "copy-engine" if self.world <= 2 else "fused"
        if factor_gather not in ("copy-engine", "fused", "nccl"):
            raise ValueError("factor_gather: 'copy-engine', 'fused' or 'nccl'")
        self.fused_gather = False
        self.fused_factors = False
        self.factor_gather = "nccl"
        self._ipc: List[Tuple[int, int]] = []
        self._push: List[Tuple[torch.cuda.Stream, int]] = []
        self._factors_pending = False
        if fused_gather is None:
            # the +/- peer stores cost the tensor-core perturbation little; the CUDA-core
            # kernel (rank > 64) stores far more per unit of its run time, and stores issued by
            # SMs to one peer drained at ~275 GB/s (70B on 2 GPUs: 12 ms added to a 14 ms
            # kernel, against ~5 ms for the NCCL all-gather), so it keeps NCCL unless asked
            fused_gather = self.aset.perturb_uses_tensor_cores
        if self.world > 1 and self.coll.stream_ordered and (fused_gather or factor_gather != "nccl"):
            self._setup_peer_gathers(fused_gather, factor_gather)

    def _setup_peer_gathers(self, fuse_pos_neg: bool, factor_mode: str) -> None:
        """Maps every peer's gather buffers into this process (CUDA IPC) for the gathers that
        move data over NVLink without NCCL:

        * +/- copies (fuse_pos_neg): the plan's perturbation stores each +/- element into
          every rank's buffer as well (byte distances handed to the plan);
        * factors, factor_mode 'fused': the update stores the bf16 shadow the same way;
          'copy-engine': gather('factors') pushes this rank's shadow into every peer's buffer
          with one device-to-device copy per peer on its own stream (copy engines, no SM).

        Every rank takes the same choice: a rank that cannot (no shadow, a failed mapping)
        makes all of them keep the NCCL all-gather."""
        import ctypes
        import torch.distributed as dist
        from ._lib import DsmzError, lib
        L = lib()
        names = []
        if fuse_pos_neg:
            names += ["pos", "neg"]
        if self.aset.shadow is not None and (factor_mode == "copy-engine" or (factor_mode == "fused" and names)):
            names.append("factors")
        ok = bool(self.aset.modules) and bool(names)
        mine = {}
        if ok:
            for name in names:
                h = ctypes.create_string_buffer(64)
                off = ctypes.c_int64(0)
                if L.dsmz_ipc_export(self.gathered[name].data_ptr(), h, ctypes.byref(off)) != 0:
                    ok = False
                    break
                mine[name] = (h.raw, off.value)
        allh = [None] * self.world
        dist.all_gather_object(allh, (ok, mine), group=self.pg)
        ok = all(x[0] for x in allh)
        deltas = {n: [] for n in names}
        if ok and any(set(x[1].keys()) != set(names) for x in allh):
            ok = False                        # every rank maps the same gathers
        if ok:
            for p in range(self.world):
                if p == self.rank:
                    continue
                for name in names:
                    h, off = allh[p][1][name]
                    ptr = ctypes.c_void_p(0)
                    if L.dsmz_ipc_import(ctypes.create_string_buffer(h, 64), off, ctypes.byref(ptr)) != 0:
                        ok = False
                        break
                    self._ipc.append((ptr.value, off))
                    deltas[name].append(ptr.value - self.gathered[name].data_ptr())
                if not ok:
                    break
        flag = torch.tensor([1 if ok else 0], dtype=torch.int32, device=self.aset.device)
        dist.all_reduce(flag, op=dist.ReduceOp.MIN, group=self.pg)
        ok = int(flag.item()) == 1
        fuse = "pos" in names
        fuse_f = fuse and factor_mode == "fused" and "factors" in names
        if ok and fuse:
            try:
                self.aset.set_gather_peers(deltas["pos"], deltas["neg"], deltas["factors"] if fuse_f else None)
            except DsmzError:
                ok = False
        flag.fill_(1 if ok else 0)
        dist.all_reduce(flag, op=dist.ReduceOp.MIN, group=self.pg)
        if int(flag.item()) == 0:
            if ok and fuse:
                self.aset.set_gather_peers([], [])
            self.close()
            return
        self.fused_gather = fuse
        self.fused_factors = fuse_f
        self._barrier = torch.zeros(1, dtype=torch.int32, device=self.aset.device)
        if "factors" in names and not fuse_f:
            # one stream per peer, so the copies run side by side on the copy engines; the
            # destination is this rank's slice of the peer's gather buffer
            self.factor_gather = "copy-engine"
            self._cstream = torch.cuda.Stream(device=self.aset.device)
            self._barrier_f = torch.zeros(2, dtype=torch.int32, device=self.aset.device)
            mine_at = self.gathered["factors"].data_ptr() + \
                self.rank * self.layout.capacity * self.gathered["factors"].element_size()
            self._push = [(torch.cuda.Stream(device=self.aset.device), mine_at + d)
                          for d in deltas["factors"]]
        elif fuse_f:
            self.factor_gather = "fused"

    def close(self) -> None:
        """Unmaps the peers' gather buffers (after the copies still in flight into them)."""
        from ._lib import lib
        if self._push:
            self._cstream.synchronize()
            self._push = []
        if self.fused_gather:
            self.aset.set_gather_peers([], [])
        self.fused_gather = False
        self.fused_factors = False
        self.factor_gather = "nccl"
        for ptr, off in self._ipc:
            lib().dsmz_ipc_close(ptr, off)
        self._ipc = []

    def calibrate(self, generator: Optional[torch.Generator] = None, niter: int = 3):
        """First-step calibration of this rank's bases (AdapterSet.calibrate) with the
        sketches the one-GPU calibration would draw: this rank's first sketch sits after
        the earlier ranks' sketches (the bases are one contiguous run of the model's basis
        order), and every rank advances the generator by the whole model's draws."""
        from .calibration import basis_draw_increments, generator_of
        gen = generator_of(self.aset.device, generator)
        layout = device_layout(self.aset.device)
        incs = [basis_draw_increments(bs, self.aset.basis_width, *layout) for bs in self.layout.rank_bases]
        start = gen.get_offset()
        before = sum(sum(x) for x in incs[: self.rank])
        total = sum(sum(x) for x in incs)
        self.aset.calibrate(generator=gen, niter=niter, offset=start + before, advance=total)

    # ------------------------------------------------------------------ phases
    def perturb(self):
        """Power iteration, perturbation, pos/neg; Kalman sums all-reduced across ranks."""
        if self.coll is not None:
            self.coll.check()                 # a collective of an earlier phase ran out of time
        if self.fused_gather:
            # the peers' stores land in every rank's +/- buffers: every rank has finished
            # reading the previous step's copies (its reads precede this on its stream)
            self.coll.all_reduce(self._barrier, "+/- buffers barrier")
        self.ctl.perturb()
        if self.world > 1:
            self.coll.all_reduce(self.aset.kalman_sums(), "Kalman sums all-reduce")

    def broadcast_dd(self, dd, src: int = 0):
        """The projected-gradient scalar(s) dd = (L+ - L-) / (2 eps) from the scoring rank
        (one float, or one per direction)."""
        one = isinstance(dd, (int, float))
        vals = [float(dd)] if one else [float(x) for x in dd]
        if self.world == 1:
            return vals[0] if one else vals
        t = torch.tensor(vals, dtype=torch.float64, device=self.aset.device)
        self.coll.check()
        self.coll.broadcast(t, src, "dd broadcast")
        self.coll.settle()                    # the value is needed on the host
        return float(t[0]) if one else t.tolist()

    def update(self, dd):
        if self.coll is not None:
            self.coll.check()
            self.coll.wait_for("factors")    # the last gather of the shadow before it is rewritten
            if self._push:                   # ... or the last copies out of it
                torch.cuda.current_stream(self.aset.device).wait_stream(self._cstream)
        self.ctl.update(dd)

    def _push_factors(self) -> None:
        """Copy-engine factor gather: after a barrier (every rank's earlier reads of its
        gathered factors are done), one copy per peer of this rank's shadow into its slice
        of the peer's buffer, each on its own stream, beside whatever the current stream runs
        next. _land_factors() orders their arrival."""
        from ._lib import check, lib
        cur = torch.cuda.current_stream(self.aset.device)
        cs = self._cstream
        cs.wait_stream(cur)                  # the update has written the shadow
        with torch.cuda.stream(cs):
            self.coll.all_reduce(self._barrier_f[:1], "factor buffers barrier")
        src = self.aset.shadow.data_ptr()
        nbytes = self.layout.sizes[self.rank] * self.aset.shadow.element_size()
        for st, dst in self._push:
            st.wait_stream(cs)
            check(lib().dsmz_peer_copy(dst, src, nbytes, st.cuda_stream), "factor copy to a peer")
        for st, _ in self._push:
            cs.wait_stream(st)
        self._factors_pending = True

    def _land_factors(self) -> None:
        """Orders every rank's factor copies into this rank's buffer on the current stream (a
        barrier after each rank's copies)."""
        if not self._factors_pending:
            return
        with torch.cuda.stream(self._cstream):
            self.coll.all_reduce(self._barrier_f[1:], "factor copies landed")
        torch.cuda.current_stream(self.aset.device).wait_stream(self._cstream)
        self._factors_pending = False

    def _arena(self, name: str) -> torch.Tensor:
        # 'factors' is what the rollout loads: the copy-dtype shadow (the fp32 masters when
        # the copy dtype is fp32)
        return self.aset.export_factors if name == "factors" else getattr(self.aset, name)

    def gather(self, *names: str):
        """All-gathers the named arenas ('factors', 'pos', 'neg') into full-model buffers
        laid out rank by rank (each rank's slice padded to the largest shard).

        'pos' and 'neg' are ordered on the current stream at once (the scoring pass needs
        them next). The 'factors' gather is left to overlap the next step's power iteration
        and perturbation, which do not touch the shadow it sends: the stream waits for it
        before the next update rewrites the shadow, or when the factors are exported. With
        copy-engine factor gathers the copies run on their own streams (no SM)."""
        if self.world == 1:
            return {n: self._arena(n) for n in names}
        self.coll.check()
        for n in names:
            if n == "factors" and self._push:
                self._push_factors()         # each peer's copies follow its earlier ones on
                continue                     # its streams, so earlier ones need no wait here
            if self.fused_gather and n in ("pos", "neg"):
                continue                     # the perturbation stored them on every rank; the
                                             # Kalman all-reduce after it ordered those stores
            if self.fused_factors and n == "factors":
                # the update stored the shadow on every rank: a stream-ordered barrier orders
                # every rank's reads after every rank's stores
                self.coll.all_reduce(self._barrier, "factor buffers barrier")
                continue
            self.coll.wait_for(n)            # a buffer still being gathered is not reused
            self.coll.all_gather_into(self.gathered[n], self._arena(n), f"{n} all-gather",
                                      defer="factors" if n == "factors" else None)
        return {n: self.gathered[n] for n in names}

    def synchronize(self) -> None:
        """Waits (bounded) for every collective and factor copy issued so far."""
        if self.coll is not None:
            self._land_factors()
            self.coll.settle()

    def full_view(self, buf: torch.Tensor, rank: int) -> torch.Tensor:
        """Rank `rank`'s factor elements inside a gathered buffer."""
        cap = self.layout.capacity
        return buf[rank * cap: rank * cap + self.layout.sizes[rank]]

    def export_adapters(self, which: str = "pos", direction: int = 0) -> Dict[str, torch.Tensor]:
        """The adapter tensors the rollout engine loads, keyed as the reference's PEFT file
        (ds_mezo/backend.py:21-36: lora_A.weight = B, lora_B.weight = A, bf16), as device
        views of the full-model buffer that the last gather(which) filled (the local arena on
        one GPU). With a bf16 copy dtype nothing is copied: this replaces the reference's bf16
        cast and safetensors write to /dev/shm. An fp32 copy dtype is converted once on the
        device into a bf16 buffer of the same layout. which: 'pos', 'neg' or 'factors'. With
        copy-engine factor gathers, export_adapters('factors') issues a collective (a barrier
        after every rank's copies): call it on every rank."""
        if which not in ("pos", "neg", "factors"):
            raise ValueError("export_adapters: which is 'pos', 'neg' or 'factors'")
        K = 1 if which == "factors" else self.aset.directions
        if not 0 <= direction < K:
            raise ValueError(f"export_adapters: direction must be in [0, {K})")
        cap = self.layout.capacity
        if self.world == 1:
            buf = self._arena(which)
        else:
            self.coll.wait_for(which)
            if which == "factors":
                self._land_factors()
            buf = self.gathered[which]
        rank_r = self._shape[4]
        idx = export_index(self.layout.rank_modules, rank_r, K * cap, direction * cap)
        if buf.dtype != torch.bfloat16:
            from ._lib import DSMZ_BF16, DSMZ_F32, check, lib
            out = torch.empty(buf.numel(), dtype=torch.bfloat16, device=buf.device)
            check(lib().dsmz_activation_load(DSMZ_BF16, out.data_ptr(), 1, buf.numel(), buf.numel(), DSMZ_F32,
                                             buf.data_ptr(), 1, buf.numel(), 1,
                                             torch.cuda.current_stream(buf.device).cuda_stream),
                  "export_adapters conversion")
            buf = out
        return {k: buf[o:o + a * b].view(a, b) for k, (o, (a, b)) in idx.items()}

