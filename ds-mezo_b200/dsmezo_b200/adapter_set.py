"""Grouped optimizer step over a whole PiSSA adapter set.

``AdapterSet`` keeps every adapter of every layer in contiguous HBM arenas, in the
controller's module order (sorted by (layer, module name), ds_mezo/model_config.py:37):

* the fp32 master factor arena (A then B of each module), as the reference keeps A and B
  in fp32 (ds_mezo/controller.py:66-67);
* what the rollout engine loads, in the copy dtype (bf16 for the bf16 configs): the +/-
  copies (the reference's fp32 pos/neg, cast at export by ds_mezo/backend.py:21-36) and,
  when the copy dtype is not fp32, a shadow of the masters rewritten by every update;
* fp32 Kalman mean (momentum) and variance arenas, and the fp32 perturbation z
  (the reference's ``perturbations`` dict, ds_mezo/controller.py:239);
* one activation buffer H (T x D) and one basis V (D x R, fp32) per unique module input
  (q/k/v share one, gate/up share one: ds_mezo/backend.py:49-52).

A layer range is one contiguous slice of every arena, so layer sharding over ranks and
the all-gather of the factors are single NCCL calls. ``ZOController`` runs the hot-path
methods of DSMeZO_Controller (ds_mezo/controller.py:165-292) on it with one grouped
launch sequence per phase.
"""
from __future__ import annotations

import ctypes
import math
from dataclasses import dataclass
from typing import List, Optional, Sequence

import torch

from . import _lib
from ._lib import DSMZ_BF16, DSMZ_F32, BasisSpec, ModuleSpec, PlanDesc, check, lib

FLT_MIN = float(torch.finfo(torch.float32).tiny)
FLT_EPS = float(torch.finfo(torch.float32).eps)
_DT = {torch.float32: DSMZ_F32, torch.bfloat16: DSMZ_BF16}

MODULE_NAMES = ("down_proj", "gate_proj", "k_proj", "o_proj", "q_proj", "up_proj", "v_proj")
INPUT_OF = {"q_proj": "qkv", "k_proj": "qkv", "v_proj": "qkv", "o_proj": "o",
            "gate_proj": "gate_up", "up_proj": "gate_up", "down_proj": "down"}
INPUT_ORDER = ("qkv", "o", "gate_up", "down")


@dataclass(frozen=True)
class ModuleShape:
    layer: int
    name: str
    d_out: int
    d_in: int
    basis: int          # index into the basis list


@dataclass(frozen=True)
class BasisShape:
    layer: int
    name: str           # module input: qkv, o, gate_up, down
    T: int              # activation rows (tokens)
    D: int              # activation width


def transformer_adapter_shapes(layers: int, hidden: int, intermediate: int, kv_out: int, tokens: int,
                               layer_range: Optional[range] = None):
    """Module and basis shapes of a Llama/Qwen-style decoder (q, k, v, o, gate, up, down)."""
    dims = {"q_proj": (hidden, hidden), "k_proj": (kv_out, hidden), "v_proj": (kv_out, hidden),
            "o_proj": (hidden, hidden), "gate_proj": (intermediate, hidden), "up_proj": (intermediate, hidden),
            "down_proj": (hidden, intermediate)}
    in_dim = {"qkv": hidden, "o": hidden, "gate_up": hidden, "down": intermediate}
    lr = range(layers) if layer_range is None else layer_range
    mods, bases = [], []
    for li in lr:
        base0 = len(bases)
        for g in INPUT_ORDER:
            bases.append(BasisShape(li, g, tokens, in_dim[g]))
        for name in MODULE_NAMES:
            d_out, d_in = dims[name]
            mods.append(ModuleShape(li, name, d_out, d_in, base0 + INPUT_ORDER.index(INPUT_OF[name])))
    return mods, bases


def device_layout(device) -> tuple:
    p = torch.cuda.get_device_properties(device)
    return p.multi_processor_count, p.max_threads_per_multi_processor


def draw_increments(modules: Sequence[ModuleShape], rank: int, basis_width: int, sm_count: int,
                    max_threads_per_sm: int) -> List[int]:
    """Generator offset advance of each module's two draws (Zc_B then Zc_A,
    ds_mezo/controller.py:184-191) on a device with the given layout."""
    L = lib()
    out = []
    rca = min(rank, basis_width)
    for m in modules:
        out.append(int(L.dsmz_randn_offset_increment(rank * basis_width, sm_count, max_threads_per_sm))
                   + int(L.dsmz_randn_offset_increment(m.d_out * rca, sm_count, max_threads_per_sm)))
    return out


class AdapterSet:
    """Arenas + bound plan for one set of modules (all of them, or one rank's layers)."""

    def __init__(self, modules: Sequence[ModuleShape], bases: Sequence[BasisShape], rank: int, basis_width: int,
                 copy_dtype=torch.float32, act_dtype=torch.bfloat16, device="cuda",
                 keep_ns_output: bool = False, rng_offset_before: int = 0, layout: Optional[tuple] = None,
                 tensor_core_power_iter: bool = True, capacity: int = 0, directions: int = 1,
                 rng_direction_stride: int = 0, single_pass_power_iter: bool = False,
                 module_rng_offsets: Optional[Sequence[int]] = None, tensor_core_perturb: bool = True,
                 pos_buffer: Optional[torch.Tensor] = None, neg_buffer: Optional[torch.Tensor] = None,
                 shadow_buffer: Optional[torch.Tensor] = None):
        if copy_dtype not in _DT or act_dtype not in _DT:
            raise ValueError("copy and activation dtypes must be float32 or bfloat16")
        self.device = torch.device(device)
        self.modules = list(modules)
        self.bases = list(bases)
        self.rank = int(rank)
        self.basis_width = int(basis_width)
        self.copy_dtype = copy_dtype
        self.act_dtype = act_dtype
        if not 1 <= int(directions) <= _lib.MAX_DIRECTIONS:
            raise ValueError(f"directions must be in [1, {_lib.MAX_DIRECTIONS}]")
        self.directions = int(directions)
        r = self.rank
        self.offA, self.offB = [], []
        n = 0
        for m in self.modules:
            self.offA.append(n)
            n += m.d_out * r
            self.offB.append(n)
            n += r * m.d_in
        self.numel = n
        # Factor arenas may be padded to `capacity` elements so that every rank of a
        # layer-sharded set sends equal-sized buffers to an all-gather.
        cap = max(n, int(capacity))
        self.capacity = cap
        dev = self.device
        K = self.directions
        self.factors = torch.zeros(cap, dtype=torch.float32, device=dev)      # fp32 masters
        # the updated factors in the copy dtype, written by every update (none for fp32)
        self.shadow = None
        if copy_dtype != torch.float32:
            self.shadow = torch.zeros(cap, dtype=copy_dtype, device=dev) if shadow_buffer is None else shadow_buffer
            if shadow_buffer is not None and (shadow_buffer.dtype != copy_dtype or shadow_buffer.numel() != cap or
                                              not shadow_buffer.is_contiguous() or shadow_buffer.device != dev):
                raise ValueError("the shadow buffer must be contiguous, of the copy dtype and hold capacity elements")
        # direction k's +/- copies and z follow direction 0's at a fixed stride
        # (or the caller's buffers: this rank's slices of the gather buffers of a sharded step)
        def copies(buf):
            if buf is None:
                return torch.zeros(K * cap, dtype=copy_dtype, device=dev)
            if buf.dtype != copy_dtype or buf.numel() != K * cap or not buf.is_contiguous() or buf.device != dev:
                raise ValueError("a +/- buffer must be contiguous, of the copy dtype and hold directions x capacity")
            return buf
        self.pos = copies(pos_buffer)
        self.neg = copies(neg_buffer)
        self.mu = torch.zeros(n, dtype=torch.float32, device=dev)
        self.var = torch.zeros(n, dtype=torch.float32, device=dev)
        self.z = torch.zeros(K * n, dtype=torch.float32, device=dev)
        self._rng_dir_stride = int(rng_direction_stride)
        self.scratch = torch.zeros(n, dtype=torch.float32, device=dev) if keep_ns_output else None
        self.offH, self.offV = [], []
        nh = nv = 0
        for b in self.bases:
            self.offH.append(nh)
            nh += b.T * b.D
            self.offV.append(nv)
            nv += b.D * self.basis_width
        self.H_arena = torch.zeros(max(nh, 1), dtype=act_dtype, device=dev)
        self.V_arena = torch.zeros(max(nv, 1), dtype=torch.float32, device=dev)
        self.layout = layout if layout is not None else device_layout(dev)
        self._flags = (0 if tensor_core_power_iter else _lib.PLAN_SIMT_POWER_ITER) | \
            (_lib.PLAN_SINGLE_PASS_POWER_ITER if single_pass_power_iter else 0) | \
            (0 if tensor_core_perturb else _lib.PLAN_CUDA_CORE_PERTURB)
        self._module_offsets = None if module_rng_offsets is None else [int(x) for x in module_rng_offsets]
        if self._module_offsets is not None and len(self._module_offsets) != len(self.modules):
            raise ValueError("module_rng_offsets needs one offset per module")
        self._build_plan(int(rng_offset_before))

    @property
    def export_factors(self) -> torch.Tensor:
        """The updated factors as the rollout loads them: the copy-dtype shadow, or the fp32
        masters themselves when the copy dtype is fp32."""
        return self.shadow if self.shadow is not None else self.factors

    def sync_shadow(self) -> None:
        """Rewrites the shadow from the masters (round to nearest even, as torch's .to()).
        Every update does this on its own; call it after writing the masters directly (the
        initial load of the adapters, a checkpoint restore). Runs on the current stream."""
        if self.shadow is None or self.numel == 0:
            return
        check(lib().dsmz_activation_load(_DT[self.copy_dtype], self.shadow.data_ptr(), 1, self.numel, self.numel,
                                         DSMZ_F32, self.factors.data_ptr(), 1, self.numel, 1, self._stream()),
              "sync_shadow")

    # ------------------------------------------------------------------ views
    def A(self, i, t=None):
        m = self.modules[i]
        return (self.factors if t is None else t)[self.offA[i]:self.offA[i] + m.d_out * self.rank].view(m.d_out, self.rank)

    def B(self, i, t=None):
        m = self.modules[i]
        return (self.factors if t is None else t)[self.offB[i]:self.offB[i] + self.rank * m.d_in].view(self.rank, m.d_in)

    def pos_dir(self, k: int) -> torch.Tensor:
        """Direction k's + copy of the factor arena."""
        return self.pos[k * self.capacity:(k + 1) * self.capacity]

    def neg_dir(self, k: int) -> torch.Tensor:
        return self.neg[k * self.capacity:(k + 1) * self.capacity]

    def z_dir(self, k: int) -> torch.Tensor:
        return self.z[k * self.numel:(k + 1) * self.numel]

    def H(self, b):
        s = self.bases[b]
        return self.H_arena[self.offH[b]:self.offH[b] + s.T * s.D].view(s.T, s.D)

    def load_activations(self, b: int, src: torch.Tensor) -> None:
        """Device-resident activation handoff for basis `b`: the module input a forward hook
        captured (n <= T rows of D features, fp32 or bf16, on this set's device, any strides)
        is converted on the device into the activation buffer H(b); rows n..T-1 become zero,
        which leaves H^T H unchanged. Replaces the reference's pinned-host round trip
        (ds_mezo/backend.py:68-93 and the .cuda() copy at ds_mezo/controller.py:171).
        Runs on the current stream."""
        s = self.bases[b]
        if src.dim() != 2 or src.shape[1] != s.D or src.shape[0] > s.T:
            raise ValueError(f"load_activations: basis {b} takes up to {s.T} rows of {s.D} features, "
                             f"got {tuple(src.shape)}")
        if src.device != self.H_arena.device:
            raise ValueError("load_activations: the source must be on the adapter set's device")
        codes = {torch.float32: DSMZ_F32, torch.bfloat16: DSMZ_BF16}
        if src.dtype not in codes:
            raise TypeError("load_activations: the source must be float32 or bfloat16")
        dst = self.H(b)
        check(lib().dsmz_activation_load(codes[self.H_arena.dtype], dst.data_ptr(), s.T, s.D, s.D,
                                         codes[src.dtype], src.data_ptr() if src.numel() else None,
                                         src.shape[0], src.stride(0), src.stride(1), self._stream()),
              "dsmz_activation_load")

    def V(self, b):
        s = self.bases[b]
        return self.V_arena[self.offV[b]:self.offV[b] + s.D * self.basis_width].view(s.D, self.basis_width)

    # ------------------------------------------------------------------ plan
    def _build_plan(self, rng_offset_before: int):
        L = lib()
        cdt = _DT[self.copy_dtype]
        fsz = self.pos.element_size()
        specs = (ModuleSpec * max(len(self.modules), 1))()
        for i, m in enumerate(self.modules):
            s = specs[i]
            a, b = self.offA[i], self.offB[i]
            s.A = self.factors.data_ptr() + a * 4
            s.B = self.factors.data_ptr() + b * 4
            if self.shadow is not None:
                s.shadow_A = self.shadow.data_ptr() + a * fsz
                s.shadow_B = self.shadow.data_ptr() + b * fsz
            s.pos_A = self.pos.data_ptr() + a * fsz
            s.pos_B = self.pos.data_ptr() + b * fsz
            s.neg_A = self.neg.data_ptr() + a * fsz
            s.neg_B = self.neg.data_ptr() + b * fsz
            s.mu_A = self.mu.data_ptr() + a * 4
            s.mu_B = self.mu.data_ptr() + b * 4
            s.var_A = self.var.data_ptr() + a * 4
            s.var_B = self.var.data_ptr() + b * 4
            s.z_A = self.z.data_ptr() + a * 4
            s.z_B = self.z.data_ptr() + b * 4
            if self.scratch is not None:
                s.scratch_A = self.scratch.data_ptr() + a * 4
                s.scratch_B = self.scratch.data_ptr() + b * 4
            s.d_out, s.d_in, s.r = m.d_out, m.d_in, self.rank
            s.ld_A, s.ld_B = self.rank, m.d_in
            s.basis, s.layer = m.basis, m.layer
        bspecs = (BasisSpec * max(len(self.bases), 1))()
        hsz = self.H_arena.element_size()
        for i, b in enumerate(self.bases):
            s = bspecs[i]
            s.H = self.H_arena.data_ptr() + self.offH[i] * hsz
            s.h_dtype = _DT[self.act_dtype]
            s.T, s.D, s.ld_H = b.T, b.D, b.D
            s.V = self.V_arena.data_ptr() + self.offV[i] * 4
            s.R = self.basis_width
        desc = PlanDesc()
        desc.copy_dtype = cdt
        desc.num_modules = len(self.modules)
        desc.modules = specs
        desc.num_bases = len(self.bases)
        desc.bases = bspecs
        desc.sm_count, desc.max_threads_per_sm = self.layout
        desc.rng_offset_before = rng_offset_before
        desc.flags = self._flags
        desc.directions = self.directions
        desc.dir_stride_factor = self.capacity
        desc.dir_stride_z = self.numel
        desc.rng_direction_stride = self._rng_dir_stride
        if self._module_offsets is not None:
            self._offsets_arr = (ctypes.c_uint64 * max(len(self._module_offsets), 1))(*self._module_offsets)
            desc.module_rng_offsets = self._offsets_arr
        handle = ctypes.c_void_p()
        check(L.dsmz_plan_create(ctypes.byref(desc), ctypes.byref(handle)), "dsmz_plan_create")
        self._plan = handle
        self.table = torch.empty(max(int(L.dsmz_plan_table_bytes(handle)), 64), dtype=torch.uint8, device=self.device)
        self.workspace = torch.empty(int(L.dsmz_plan_workspace_bytes(handle)), dtype=torch.uint8, device=self.device)
        self.rng_increment = int(L.dsmz_plan_rng_increment(handle))
        check(L.dsmz_plan_bind(handle, self.table.data_ptr(), self.table.numel(), self.workspace.data_ptr(),
                               self.workspace.numel(), self._stream()), "dsmz_plan_bind")
        addr = L.dsmz_step_kalman_sums(handle)
        off = addr - self.workspace.data_ptr()
        self._kal = self.workspace[off:off + 16 * self.directions].view(torch.float64)
        self.launches = 0            # kernels this set has launched
        self._v_version = None       # basis arena version after the last power iteration

    def __del__(self):
        h = getattr(self, "_plan", None)
        if h is not None and h.value:
            try:
                lib().dsmz_plan_destroy(h)
            except Exception:
                pass
            self._plan = None

    def _stream(self):
        return torch.cuda.current_stream(self.device).cuda_stream

    @property
    def uses_tensor_cores(self) -> bool:
        """True when the power iteration runs on tcgen05 tensor cores."""
        return bool(lib().dsmz_plan_uses_tensor_cores(self._plan))

    @property
    def single_pass_power_iter(self) -> bool:
        """True when each power iteration reads every activation from HBM once (the W
        product re-reads each token tile from L2 right after the Y product streamed it)."""
        return int(lib().dsmz_plan_uses_tensor_cores(self._plan)) == 2

    def device_error(self) -> int:
        """Reads and clears the device error word (synchronises the stream)."""
        return int(lib().dsmz_plan_device_error(self._plan, self._stream()))

    def factor_norms(self) -> torch.Tensor:
        """Frobenius norms of the fp32 masters, A then B of each module (device, fp32)."""
        out = torch.empty(2 * len(self.modules), dtype=torch.float32, device=self.device)
        if self.modules:
            check(lib().dsmz_plan_factor_norms(self._plan, out.data_ptr(), self._stream()), "factor norms")
            self.launches += 2
        return out

    def launch_count(self, num_iters: int) -> int:
        return int(lib().dsmz_plan_launch_count(self._plan, num_iters))

    # ------------------------------------------------------------------ phases
    def power_iteration(self, num_iters: int = 3, norm_floor: float = FLT_MIN):
        """Power iteration of every basis. When no basis was written since this set's last
        power iteration (torch's version counter of the basis arena is unchanged: the
        library's own writes do not move it), the tensor-core path reuses that iteration's
        bf16 split of the bases."""
        unchanged = self._v_version is not None and self._v_version == self.V_arena._version
        flags = _lib.PI_BASIS_UNCHANGED if unchanged else 0
        check(lib().dsmz_step_power_iteration_ex(self._plan, int(num_iters), float(norm_floor), flags,
                                                 self._stream()), "power iteration")
        n = self.launch_count(num_iters) - self.launch_count(0)
        self.launches += n - (1 if (unchanged and self.uses_tensor_cores and num_iters > 0) else 0)
        self._v_version = self.V_arena._version if num_iters > 0 else self._v_version

    def calibrate(self, generator: Optional[torch.Generator] = None, niter: int = 3, norm_floor: float = FLT_MIN,
                  offset: Optional[int] = None, advance: Optional[int] = None,
                  singular_values: bool = False) -> Optional[torch.Tensor]:
        """First-step calibration (ds_mezo/controller.py:156-163): every basis becomes V of
        torch.svd_lowrank(H, q=basis_width, niter) of its loaded activation, the sketches
        drawn in basis order from `generator` (default: the device's default CUDA generator,
        which svd_lowrank uses). `offset`: the generator offset of this set's first sketch
        (default: the generator's current offset); `advance`: how far to move the generator
        afterwards (default: this set's draws). Returns the Ritz singular values
        (num_bases x basis_width) when asked."""
        from .calibration import generator_of
        L = lib()
        gen = generator_of(self.device, generator)
        seed = gen.initial_seed()
        off = gen.get_offset() if offset is None else int(offset)
        start = gen.get_offset()
        inc = int(L.dsmz_plan_calibration_rng_increment(self._plan))
        nbytes = int(L.dsmz_plan_calibration_workspace_bytes(self._plan))
        ws = torch.empty(nbytes, dtype=torch.uint8, device=self.device)
        sv = torch.empty((len(self.bases), self.basis_width), dtype=torch.float32, device=self.device) \
            if singular_values else None
        check(L.dsmz_plan_calibrate(self._plan, int(seed) & (2 ** 64 - 1), off, int(niter), float(norm_floor),
                                    ws.data_ptr(), nbytes, sv.data_ptr() if sv is not None else None,
                                    self._stream()), "calibration")
        ws.record_stream(torch.cuda.current_stream(self.device))
        gen.set_offset(start + (inc if advance is None else int(advance)))
        self.launches += int(L.dsmz_plan_calibration_launch_count(self._plan, int(niter)))
        self._v_version = None
        return sv

    @property
    def perturb_uses_tensor_cores(self) -> bool:
        return bool(lib().dsmz_plan_perturb_on_tensor_cores(self._plan))

    def set_gather_peers(self, pos_deltas: Sequence[int], neg_deltas: Sequence[int],
                         shadow_deltas: Optional[Sequence[int]] = None):
        """Byte distances from this set's +/- buffers (and factor shadow) to each peer's
        mapped buffers: the perturbation (and the update) store every element there too
        (dsmz_plan_set_gather_peers)."""
        n = len(pos_deltas)
        pa = (ctypes.c_int64 * max(n, 1))(*[int(x) for x in pos_deltas])
        na = (ctypes.c_int64 * max(n, 1))(*[int(x) for x in neg_deltas])
        sa = (ctypes.c_int64 * max(n, 1))(*[int(x) for x in shadow_deltas]) if shadow_deltas else None
        check(lib().dsmz_plan_set_gather_peers(self._plan, n, pa, na, sa), "gather peers")

    def calibration_launch_count(self, niter: int = 3) -> int:
        return int(lib().dsmz_plan_calibration_launch_count(self._plan, int(niter)))

    def draw(self, seed: int, offset: int):
        """Issue the perturbation's Zc_A draws ahead, on the current stream (dsmz_step_draw);
        the next perturb with the same seed and offset uses them."""
        check(lib().dsmz_step_draw(self._plan, int(seed) & (2 ** 64 - 1), int(offset), self._stream()), "draws")

    def perturb(self, seed: int, offset: int, eps: float, beta: float, q: float, norm_floor: float = FLT_MIN):
        check(lib().dsmz_step_perturb(self._plan, int(seed) & (2 ** 64 - 1), int(offset), float(eps), float(beta),
                                      float(q), float(norm_floor), self._stream()), "perturbation")
        self.launches += 1 + 4 * self.directions if self.numel else 0

    def kalman_sums(self) -> torch.Tensor:
        """Device view of the rank-local (sum z*mu1, sum z^2*var1) of every direction
        (2 doubles per direction); all-reduce it in place."""
        return self._kal

    def update(self, dd, beta: float, q: float, eta: float, norm_floor: float = FLT_MIN, schedule="cubic"):
        """dd: the projected-gradient scalar (one direction) or one per direction."""
        sched = _lib.schedule(schedule)
        dds = [float(dd)] if isinstance(dd, (int, float)) else [float(x) for x in dd]
        if len(dds) != self.directions:
            raise ValueError(f"need {self.directions} projected-gradient scalars, got {len(dds)}")
        if self.directions == 1:
            check(lib().dsmz_step_update(self._plan, dds[0], float(beta), float(q), float(eta), float(norm_floor),
                                         sched, self._stream()), "update")
            self.launches += 3 if self.numel else 0
            return
        arr = (ctypes.c_float * len(dds))(*dds)
        check(lib().dsmz_step_update_directions(self._plan, arr, len(dds), float(beta), float(q), float(eta),
                                                float(norm_floor), sched, self._stream()), "update")
        self.launches += 4 if self.numel else 0


def rloo_direction_scalars(rewards: torch.Tensor, eps: float) -> List[float]:
    """Projected-gradient scalars of K directions from their rollout rewards.

    rewards: (K, N) with the first N/2 rollouts of each direction scored under its + copy
    and the rest under its - copy. Each rollout's advantage is its reward minus the RLOO
    baseline of its direction, (sum - r) / (N - 1); the loss of a copy is minus the mean
    advantage of its rollouts, and dd_k = (L+ - L-) / (2 eps) as in
    ds_mezo/controller.py:307 (no reference counterpart for K > 1: the reference scores
    one direction per step with shrinkage RLOO)."""
    r = rewards.double()
    K, N = r.shape
    if N < 2 or N % 2:
        raise ValueError("need an even number (>= 2) of rollouts per direction")
    base = (r.sum(dim=1, keepdim=True) - r) / (N - 1)
    adv = r - base
    lp = -adv[:, : N // 2].mean(dim=1)
    lm = -adv[:, N // 2:].mean(dim=1)
    return ((lp - lm) / (2.0 * eps)).tolist()


def eps_from_norms(norms: torch.Tensor) -> float:
    """The perturbation scale of ds_mezo/controller.py:78-82 from every factor's Frobenius
    norm: torch.median (the lower middle value of an even count) times FLT_EPSILON^(1/3)."""
    v = sorted(float(x) for x in norms.detach().cpu().tolist())
    if not v:
        raise ValueError("eps_from_norms: no factors")
    return v[(len(v) - 1) // 2] * FLT_EPS ** (1.0 / 3.0)


class ShrinkageRLOO:
    """Advantages of one step's rollouts with the James-Stein shrinkage of the RLOO baseline
    (ds_mezo/controller.py:216-229): with r_bar the mean reward and v the unbiased reward
    variance, lam = v / (v + (r_bar - ema)^2 + FLT_MIN), the baseline of rollout i is
    (1 - lam) * (sum - r_i) / (N - 1) + lam * ema, and afterwards
    ema <- beta * ema + (1 - beta) * r_bar with beta the Kalman momentum of the previous
    update (0 before the first). The arithmetic follows the reference's: float32 tensors for
    the rewards, Python floats for the scalars."""

    def __init__(self, norm_floor: float = FLT_MIN):
        self.reward_ema = 0.0
        self.norm_floor = float(norm_floor)

    def advantages(self, rewards: Sequence[float], momentum: float) -> List[float]:
        r = torch.tensor([float(x) for x in rewards], dtype=torch.float32)
        n = r.numel()
        if n < 2:
            raise ValueError("shrinkage RLOO needs at least two rollouts")
        r_bar = float(r.mean())
        base_rloo = (r.sum() - r) / (n - 1)
        rvar = float(r.var())
        lam = rvar / (rvar + (r_bar - self.reward_ema) ** 2 + self.norm_floor)
        base = (1.0 - lam) * base_rloo + lam * self.reward_ema
        adv = (r - base).tolist()
        self.reward_ema = momentum * self.reward_ema + (1.0 - momentum) * r_bar
        return adv


def kalman_beta_q(step_count: int, total_steps: int, eps: float):
    """ds_mezo/controller.py:255-258."""
    beta = 1.0 - 1.0 / min(step_count, int(math.sqrt(total_steps)))
    return beta, eps ** 2 * (1.0 - beta * beta)


class ZOController:
    """Hot path of DSMeZO_Controller (ds_mezo/controller.py:165-292) on an AdapterSet.

    ``perturb()`` = _update_activation_bases + _get_perturbation for every module +
    fused_perturb_dual (controller.py:236-251), drawing from ``generator`` exactly like
    the reference's per-module torch.randn calls and advancing it by the same amount.
    ``update(dd)`` = _update_weights + _step_lr (controller.py:253-292).
    With a process group the set holds this rank's layers; the two Kalman sums are
    all-reduced between the phases.
    """

    @classmethod
    def from_factors(cls, aset: AdapterSet, total_steps: int, generator: torch.Generator, **kw) -> "ZOController":
        """A controller whose eps is derived from the set's masters as the reference's
        constructor does (ds_mezo/controller.py:78-82): median factor norm times
        FLT_EPSILON^(1/3). With a process group the per-matrix norms of every rank are
        gathered (a few KB), so every rank derives the same eps."""
        norms = aset.factor_norms()
        pg = kw.get("process_group")
        if pg is not None:
            import torch.distributed as dist
            world = dist.get_world_size(pg)
            n = torch.tensor([norms.numel()], dtype=torch.int64, device=norms.device)
            counts = [torch.zeros_like(n) for _ in range(world)]
            dist.all_gather(counts, n, group=pg)
            top = int(max(int(c.item()) for c in counts))
            pad = torch.full((top,), float("nan"), dtype=torch.float32, device=norms.device)
            pad[:norms.numel()] = norms
            parts = [torch.empty_like(pad) for _ in range(world)]
            dist.all_gather(parts, pad, group=pg)
            norms = torch.cat([p[:int(c.item())] for p, c in zip(parts, counts)])
        return cls(aset, eps_from_norms(norms), total_steps, generator, **kw)

    def __init__(self, aset: AdapterSet, eps: float, total_steps: int, generator: torch.Generator,
                 power_iters: int = 3, schedule="cubic", process_group=None, rng_increment_total: Optional[int] = None,
                 norm_floor: float = FLT_MIN, overlap_draws: bool = True):
        self.aset = aset
        self.overlap_draws = bool(overlap_draws)   # Zc_A draws on a side stream beside the power iteration
        self._side = None
        self.eps = float(eps)
        self.total_steps = int(total_steps)
        self.gen = generator
        self.power_iters = int(power_iters)
        self.schedule = schedule
        self.pg = process_group
        self.norm_floor = norm_floor
        self.rng_increment_total = aset.rng_increment if rng_increment_total is None else int(rng_increment_total)
        self.step_count = 0
        self.eta_max = self.eps
        self.eta_min = self.eta_max * FLT_EPS ** (1.0 / 3.0)
        self.eta = self.eta_max
        self.beta = 0.0
        self.q = 0.0
        self.rloo = ShrinkageRLOO(norm_floor)

    def _step_lr(self):
        t = self.step_count
        self.eta = self.eta_min + 0.5 * (self.eta_max - self.eta_min) * (1.0 + math.cos(math.pi * t / self.total_steps))

    def advantages(self, rewards: Sequence[float]) -> List[float]:
        """Shrinkage-RLOO advantages of this step's rollout rewards (ds_mezo/controller.py:
        216-229). Call it before perturb(), as the reference's _explore precedes
        _perturb_and_sync: the reward EMA then moves with the previous update's momentum."""
        return self.rloo.advantages(rewards, self.beta)

    def skip(self):
        """A step whose advantages are all zero (ds_mezo/controller.py:299-301): the step count
        and the learning rate move on, nothing else does."""
        self.step_count += 1
        self._step_lr()

    def perturb(self):
        self.step_count += 1
        self.beta, self.q = kalman_beta_q(self.step_count, self.total_steps, self.eps)
        seed = self.gen.initial_seed()
        off = self.gen.get_offset()
        self.gen.set_offset(off + self.rng_increment_total)
        if self.overlap_draws and self.aset.modules and self.aset.bases:
            # the Zc_A draws depend on nothing the step computes: they run on a side stream
            # beside the (memory-bound) power iteration
            main = torch.cuda.current_stream(self.aset.device)
            if self._side is None:
                self._side = torch.cuda.Stream(device=self.aset.device)
            self._side.wait_stream(main)
            with torch.cuda.stream(self._side):
                self.aset.draw(seed, off)
            self.aset.power_iteration(self.power_iters, self.norm_floor)
            main.wait_stream(self._side)
        else:
            self.aset.power_iteration(self.power_iters, self.norm_floor)
        self.aset.perturb(seed, off, self.eps, self.beta, self.q, self.norm_floor)
        if self.pg is not None:
            from .sharding import allreduce_sums
            allreduce_sums(self.aset.kalman_sums(), self.pg)

    def update(self, dd):
        """dd: one projected-gradient scalar, or one per direction."""
        self.aset.update(dd, self.beta, self.q, self.eta, self.norm_floor, self.schedule)
        self._step_lr()
