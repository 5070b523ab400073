"""The C ABI without a GPU: the library loads, exports every function include/dsmezo.h
declares, and its host-only entry points (schedules, torch generator layout, plan
validation and layout) behave. No CUDA calls are made."""
import ctypes
import math
import re
from pathlib import Path

import pytest
import torch

from oracle import reference_ops as ref

ROOT = Path(__file__).resolve().parents[1]


@pytest.fixture(scope="module")
def L():
    from dsmezo_b200 import build
    build.build()
    from dsmezo_b200 import _lib
    return _lib.lib()


def declared_functions():
    text = (ROOT / "include" / "dsmezo.h").read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    names = re.findall(r"\b(dsmz_[a-z0-9_]+)\s*\(", text)
    return sorted(set(names))


def test_every_declared_symbol_is_exported(L):
    from dsmezo_b200 import _lib
    names = declared_functions()
    assert len(names) >= 25
    for n in names:
        assert hasattr(L, n), n
    assert set(names) == set(_lib.SIGNATURES), "ctypes signatures must mirror the header"


def test_abi_version(L):
    from dsmezo_b200._lib import ABI_VERSION
    assert L.dsmz_abi_version() == ABI_VERSION == 3


def test_cubic_schedule_matches_reference(L):
    from dsmezo_b200 import _lib
    s = _lib.schedule("cubic")
    want = ref.ns_cubic_schedule()
    assert s.iters == len(want) == 12
    for i, (c1, c3, c5) in enumerate(want):
        assert s.c[i][0] == c1 and s.c[i][1] == c3 and s.c[i][2] == 0.0
    q = _lib.schedule("quintic")
    assert q.iters == 5 and tuple(q.c[0]) == (3.4445, -4.7750, 2.0315)
    with pytest.raises(ValueError):
        _lib.schedule("septic")


def _torch_policy(n, sm, mt):
    """ATen DistributionTemplates.h calc_execution_policy with unroll 4."""
    block = 256
    grid = (n + block - 1) // block
    grid = min(sm * (mt // block), grid)
    return ((n - 1) // (block * grid * 4) + 1) * 4, grid * block


@pytest.mark.parametrize("n", [1, 2, 255, 256, 257, 303104, 303105, 1212416, 1212417, 10 ** 8])
@pytest.mark.parametrize("sm,mt", [(148, 2048), (132, 2048), (80, 1024)])
def test_generator_layout(L, n, sm, mt):
    inc, thr = _torch_policy(n, sm, mt)
    assert L.dsmz_randn_threads(n, sm, mt) == thr
    assert L.dsmz_randn_offset_increment(n, sm, mt) == inc
    assert L.dsmz_randn_offset_increment(0, sm, mt) == 0


def _bases(rank, layers=2, hidden=64, inter=176, kv=16, tokens=48):
    from dsmezo_b200 import transformer_adapter_shapes
    return transformer_adapter_shapes(layers, hidden, inter, kv, tokens)[1]


def _fake_set(layers=2, hidden=64, inter=176, kv=16, rank=8, tokens=48, bad=None, h_dtype=1):
    from dsmezo_b200 import _lib, transformer_adapter_shapes
    mods, bases = transformer_adapter_shapes(layers, hidden, inter, kv, tokens)
    specs = (_lib.ModuleSpec * len(mods))()
    fake = 0x10000
    for i, m in enumerate(mods):
        s = specs[i]
        for f in ("A", "B", "pos_A", "pos_B", "neg_A", "neg_B", "mu_A", "mu_B", "var_A", "var_B", "z_A", "z_B"):
            setattr(s, f, fake)
        s.d_out, s.d_in, s.r, s.ld_A, s.ld_B, s.basis, s.layer = m.d_out, m.d_in, rank, rank, m.d_in, m.basis, m.layer
    bs = (_lib.BasisSpec * len(bases))()
    for i, b in enumerate(bases):
        bs[i].H, bs[i].h_dtype, bs[i].T, bs[i].D, bs[i].ld_H, bs[i].V, bs[i].R = fake, h_dtype, b.T, b.D, b.D, fake, rank
    if bad == "rank":
        specs[3].r = 200
    if bad == "basis":
        specs[0].basis = 99
    if bad == "null":
        specs[1].mu_B = None
    d = _lib.PlanDesc()
    d.copy_dtype, d.num_modules, d.modules = 1, len(mods), specs
    d.num_bases, d.bases, d.sm_count, d.max_threads_per_sm = len(bases), bs, 148, 2048
    return mods, d


@pytest.mark.parametrize("rank,h_dtype,flags,path", [(8, 1, 0, 0), (16, 1, 0, 1), (16, 0, 0, 0), (64, 1, 0, 1),
                                                      (64, 1, 2, 2), (16, 1, 2, 2), (128, 1, 2, 1), (16, 0, 2, 0)])
def test_plan_create_host_only(L, rank, h_dtype, flags, path):
    from dsmezo_b200 import draw_increments
    mods, d = _fake_set(rank=rank, h_dtype=h_dtype)
    d.flags = flags
    h = ctypes.c_void_p()
    assert L.dsmz_plan_create(ctypes.byref(d), ctypes.byref(h)) == 0
    try:
        assert L.dsmz_plan_table_bytes(h) > 0 and L.dsmz_plan_workspace_bytes(h) > 0
        assert L.dsmz_plan_rng_increment(h) == sum(draw_increments(mods, rank, rank, 148, 2048))
        # tcgen05 power iteration for bf16 activations and R a multiple of 16: two products per
        # iteration, or one pass over the activations (R <= 64) when the flag asks for it
        assert L.dsmz_plan_uses_tensor_cores(h) == path
        per_iter = {0: 5, 1: 5, 2: 4}[path]
        assert L.dsmz_plan_launch_count(h, 3) == 3 * per_iter + (1 if path else 0) + 8
        # calibration: 2 sketches, niter + 2 Y products, niter + 1 W tails of 4 launches, 2 Grams
        # of Y, 2 eigen-solves, the rotation, the first bf16 split on the tensor-core path
        tcs = 1 if path else 0
        assert L.dsmz_plan_calibration_launch_count(h, 3) == 2 + 5 + 16 + 5 + tcs
        assert L.dsmz_plan_calibration_launch_count(h, 0) == 2 + 2 + 4 + 5 + tcs
        assert L.dsmz_plan_calibration_workspace_bytes(h) > 0
        assert L.dsmz_plan_calibration_rng_increment(h) == sum(
            int(L.dsmz_randn_offset_increment((b.D if b.T >= b.D else b.T) * rank, 148, 2048)) for b in _bases(rank))
        # stepping an unbound plan is an error, not a launch
        assert L.dsmz_step_update(h, 0.0, 0.0, 0.0, 0.0, 0.0, None, None) == 1
        assert b"not bound" in L.dsmz_last_error()
    finally:
        L.dsmz_plan_destroy(h)


@pytest.mark.parametrize("bad,msg", [("rank", b"invalid shape"), ("basis", b"basis index"), ("null", b"null")])
def test_plan_create_rejects(L, bad, msg):
    _, d = _fake_set(bad=bad)
    h = ctypes.c_void_p()
    assert L.dsmz_plan_create(ctypes.byref(d), ctypes.byref(h)) == 1
    assert msg in L.dsmz_last_error()


def test_dropin_argument_errors_without_gpu(L):
    # size checks happen before any CUDA call
    rc = L.dsmz_zo_muon_update(0, 0x1000, 300, 1, 0x1000, 300, 1, None, 0, 0, 1000, 300, 0.1, 1e-38, None,
                               0x1000, 1 << 20, None)
    assert rc == 4 and b"min(M, N)" in L.dsmz_last_error()
    rc = L.dsmz_zo_muon_update(0, 0x1000, 8, 1, 0x2000, 1, 8, None, 0, 0, 100, 8, 0.1, 1e-38, None,
                               0x1000, 1 << 20, None)
    assert rc == 1 and b"strides" in L.dsmz_last_error()
    rc = L.dsmz_power_iter(0, 0x1000, 10, 10, 10, 1, 0x1000, 200, 200, 1, 0x1000, 3, 1e-38, 0x1000, 1 << 20, None)
    assert rc == 4
    assert L.dsmz_zo_muon_update_workspace_bytes(18944, 64) > 0
    assert L.dsmz_power_iter_workspace_bytes(4096, 3584, 64) >= 4096 * 64 * 4 + 3584 * 64 * 4


def test_rloo_direction_scalars_match_oracle():
    from dsmezo_b200 import rloo_direction_scalars
    g = torch.Generator().manual_seed(4)
    r = torch.bernoulli(torch.full((16, 8), 0.4), generator=g)
    ours = rloo_direction_scalars(r, 1e-3)
    want = ref.rloo_direction_scalars(r, 1e-3)
    assert len(ours) == 16
    for a, b in zip(ours, want):
        assert math.isclose(a, b, rel_tol=1e-12, abs_tol=1e-9)
    # equal rewards under both copies: no signal
    assert rloo_direction_scalars(torch.ones(2, 8), 1e-3) == [0.0, 0.0]
    with pytest.raises(ValueError):
        rloo_direction_scalars(torch.ones(2, 7), 1e-3)


@pytest.mark.parametrize("K", [2, 16])
def test_plan_directions_host_only(L, K):
    from dsmezo_b200 import draw_increments
    mods, d = _fake_set(rank=16)
    d.directions, d.dir_stride_factor, d.dir_stride_z = K, 1 << 20, 1 << 20
    h = ctypes.c_void_p()
    assert L.dsmz_plan_create(ctypes.byref(d), ctypes.byref(h)) == 0
    try:
        assert L.dsmz_plan_directions(h) == K
        assert L.dsmz_plan_rng_increment(h) == K * sum(draw_increments(mods, 16, 16, 148, 2048))
        # B-side sums once, 4 launches per direction, 4 update launches
        assert L.dsmz_plan_launch_count(h, 3) == (3 * 5 + 1) + 1 + 4 * K + 4
        dd = (ctypes.c_float * K)(*([0.0] * K))
        assert L.dsmz_step_update_directions(h, dd, K, 0.0, 0.0, 0.0, 0.0, None, None) == 1   # not bound
    finally:
        L.dsmz_plan_destroy(h)
    d.dir_stride_z = 0
    assert L.dsmz_plan_create(ctypes.byref(d), ctypes.byref(h)) == 1
    assert b"direction strides" in L.dsmz_last_error()
    d.directions = 33
    assert L.dsmz_plan_create(ctypes.byref(d), ctypes.byref(h)) == 1


def test_activation_load_argument_errors_without_gpu(L):
    # every check of the activation handoff happens before any CUDA call
    assert L.dsmz_activation_load(1, None, 16, 8, 8, 0, 0x1000, 16, 8, 1, None) == 1
    assert b"null" in L.dsmz_last_error()
    assert L.dsmz_activation_load(1, 0x1000, 16, 8, 8, 0, 0x1000, 17, 8, 1, None) == 1   # n > T
    assert L.dsmz_activation_load(1, 0x1000, 16, 8, 4, 0, 0x1000, 16, 8, 1, None) == 1   # ld < D
    assert L.dsmz_activation_load(2, 0x1000, 16, 8, 8, 0, 0x1000, 16, 8, 1, None) == 1   # bad dtype
    assert b"dtypes" in L.dsmz_last_error()
    assert L.dsmz_activation_load(1, 0x1000, 16, 8, 8, 0, 0x1000, 16, -8, 1, None) == 1  # negative stride


def test_contrastive_loss_argument_errors_without_gpu(L):
    # host-side validation runs before any CUDA call
    i64 = ctypes.c_int64 * 3
    f64 = ctypes.c_double * 2
    ws = 1 << 20
    ok_start, adv = i64(0, 3, 5), f64(0.5, -0.5)
    assert L.dsmz_contrastive_loss(1, 0x1000, 50, 50, 0x2000, 5, ok_start, adv, 0, 0x3000, 0x4000, ws, None) == 1
    assert L.dsmz_contrastive_loss(7, 0x1000, 50, 50, 0x2000, 5, ok_start, adv, 2, 0x3000, 0x4000, ws, None) == 1
    assert b"kind" in L.dsmz_last_error()
    assert L.dsmz_contrastive_loss(1, 0x1000, 50, 50, 0x2000, 5, i64(1, 3, 5), adv, 2, 0x3000, 0x4000, ws, None) == 1
    assert L.dsmz_contrastive_loss(1, 0x1000, 50, 50, 0x2000, 5, i64(0, 0, 5), adv, 2, 0x3000, 0x4000, ws, None) == 1
    assert b"scored token" in L.dsmz_last_error()
    assert L.dsmz_contrastive_loss(1, 0x1000, 50, 40, 0x2000, 5, ok_start, adv, 2, 0x3000, 0x4000, ws, None) == 1
    assert L.dsmz_contrastive_loss(1, 0x1000, 50, 50, 0x2000, 5, ok_start, adv, 2, 0x3000, 0x4000, 16, None) == 2
    assert L.dsmz_contrastive_loss_workspace_bytes(1000) >= 8000
