"""GPU parity of the device-resident activation handoff (dsmz_activation_load) through the
C ABI: bit-exact against torch's own conversion on the GPU (.to(torch.bfloat16), rounding
to nearest even), on the vector and element paths, strided sources, short
captures (rows past the capture are zero) and the 7B down-projection input shape. The
AdapterSet handoff must give the same basis as writing H directly."""
import pytest
import torch

pytestmark = pytest.mark.gpu
DEV = "cuda"
F32, BF16 = 0, 1
CODE = {torch.float32: F32, torch.bfloat16: BF16}


@pytest.fixture(scope="module")
def L():
    from dsmezo_b200 import _lib
    return _lib.lib()


def load(L, dst, src, n=None):
    T, D = dst.shape
    n = src.shape[0] if n is None else n
    rc = L.dsmz_activation_load(CODE[dst.dtype], dst.data_ptr(), T, D, dst.stride(0), CODE[src.dtype],
                                src.data_ptr() if src.numel() else None, n, src.stride(0), src.stride(1),
                                torch.cuda.current_stream().cuda_stream)
    assert rc == 0, L.dsmz_last_error()


def want(src, T, dtype):
    out = torch.zeros(T, src.shape[1], dtype=dtype, device=DEV)
    out[:src.shape[0]] = src.to(dtype)
    return out


def same_bits(a, b):
    assert a.dtype == b.dtype and a.shape == b.shape
    it = torch.int16 if a.dtype == torch.bfloat16 else torch.int32
    ab, bb = a.reshape(-1).view(it), b.reshape(-1).view(it)
    bad = (ab != bb).nonzero().flatten()[:8].tolist()
    assert not bad, [(i, float(a.reshape(-1)[i]), int(ab[i]), float(b.reshape(-1)[i]), int(bb[i])) for i in bad]
    return True


def specials(n, d, gen):
    x = torch.randn(n, d, generator=gen) * torch.exp(torch.randn(n, d, generator=gen) * 3)
    flat = x.view(-1)
    vals = [0.0, -0.0, float("inf"), float("-inf"), float("nan"), 1e-40, -1e-42, 3.4e38, -3.4e38,
            1.00390625, 1.01171875, -1.00390625, 1.0 + 2 ** -8 + 2 ** -20]   # ties and near-ties
    flat[:len(vals)] = torch.tensor(vals)
    return x


@pytest.mark.parametrize("T,D,n", [(256, 3584, 256), (300, 64, 123), (33, 8, 0), (64, 520, 64)])
def test_f32_to_bf16_vector_path(L, T, D, n):
    gen = torch.Generator().manual_seed(T * 7 + D)
    src = specials(n, D, gen).to(DEV) if n else torch.empty(0, D, device=DEV)
    dst = torch.full((T, D), 7.0, dtype=torch.bfloat16, device=DEV)   # stale contents
    load(L, dst, src)
    torch.cuda.synchronize()
    assert same_bits(dst, want(src, T, torch.bfloat16))


@pytest.mark.parametrize("T,D,n", [(200, 77, 150), (17, 3, 17)])
def test_f32_to_bf16_element_path(L, T, D, n):
    gen = torch.Generator().manual_seed(D)
    src = specials(n, D, gen).to(DEV)
    dst = torch.full((T, D), -3.0, dtype=torch.bfloat16, device=DEV)
    load(L, dst, src)
    torch.cuda.synchronize()
    assert same_bits(dst, want(src, T, torch.bfloat16))


def test_strided_and_transposed_sources(L):
    gen = torch.Generator().manual_seed(5)
    base = torch.randn(512, 1200, generator=gen).to(DEV)
    cols = base[:, 16:16 + 1024]          # row pitch 1200 floats (4800 B), 64-byte offset: vector path
    dst = torch.empty(600, 1024, dtype=torch.bfloat16, device=DEV)
    load(L, dst, cols)
    tr = torch.randn(256, 384, generator=gen).to(DEV).t()   # column stride 384: element path
    dst2 = torch.empty(400, 256, dtype=torch.bfloat16, device=DEV)
    load(L, dst2, tr)
    torch.cuda.synchronize()
    assert same_bits(dst, want(cols, 600, torch.bfloat16))
    assert same_bits(dst2, want(tr, 400, torch.bfloat16))


@pytest.mark.parametrize("sdt,ddt", [(torch.bfloat16, torch.bfloat16), (torch.bfloat16, torch.float32),
                                     (torch.float32, torch.float32)])
def test_other_dtype_pairs(L, sdt, ddt):
    gen = torch.Generator().manual_seed(11)
    for T, D, n in [(128, 896, 100), (50, 13, 50)]:
        src = specials(n, D, gen).to(sdt).to(DEV)
        dst = torch.full((T, D), 9.0, dtype=ddt, device=DEV)
        load(L, dst, src)
        torch.cuda.synchronize()
        assert same_bits(dst, want(src, T, ddt))


def test_pitched_destination(L):
    # the destination may be a column window of a wider buffer (row pitch > D)
    gen = torch.Generator().manual_seed(2)
    src = torch.randn(64, 256, generator=gen).to(DEV)
    wide = torch.full((80, 320), 5.0, dtype=torch.bfloat16, device=DEV)
    dst = wide[:, 32:32 + 256]
    load(L, dst, src)
    torch.cuda.synchronize()
    assert same_bits(dst.contiguous(), want(src, 80, torch.bfloat16))
    assert torch.all(wide[:, :32] == 5.0) and torch.all(wide[:, 288:] == 5.0)   # nothing outside D touched


def test_down_projection_shape(L):
    # the 7B down-projection input: 4096 tokens x 18944 features, fp32 capture -> bf16 buffer
    gen = torch.Generator(device=DEV).manual_seed(3)
    src = torch.randn(4096, 18944, generator=gen, device=DEV)
    dst = torch.empty(4096, 18944, dtype=torch.bfloat16, device=DEV)
    load(L, dst, src)
    torch.cuda.synchronize()
    assert same_bits(dst, src.to(torch.bfloat16))


def test_adapter_set_handoff_gives_the_same_basis():
    # a forward hook's fp32 capture (shorter than the buffer) handed over on the device must
    # give the bases that writing the rounded capture into H by hand gives
    from dsmezo_b200 import AdapterSet
    from step_harness import make_inputs
    mods, bases, A, B, V0, H = make_inputs(1, 256, 704, 64, 16, 512, 21, torch.bfloat16, torch.bfloat16)
    sets = []
    for way in ("handoff", "direct"):
        aset = AdapterSet(mods, bases, 16, 16, copy_dtype=torch.bfloat16, act_dtype=torch.bfloat16, device=DEV)
        for i in range(len(mods)):
            aset.A(i).copy_(A[i])
            aset.B(i).copy_(B[i])
        gen = torch.Generator(device=DEV).manual_seed(4)
        for b in range(len(bases)):
            aset.V(b).copy_(V0[b])
            T, D = aset.H(b).shape
            cap = torch.randn(T - 37, D, generator=gen, device=DEV) * 3    # fp32 capture, 37 rows short
            aset.H(b).fill_(1.0)                                            # stale contents
            if way == "handoff":
                aset.load_activations(b, cap)
            else:
                aset.H(b).zero_()
                aset.H(b)[:T - 37] = cap.to(torch.bfloat16)
        aset.power_iteration(3)
        sets.append(aset)
    torch.cuda.synchronize()
    assert sets[0].device_error() == 0
    assert torch.equal(sets[0].H_arena, sets[1].H_arena)
    assert torch.equal(sets[0].V_arena, sets[1].V_arena)


def test_adapter_set_handoff_rejects_bad_sources():
    from dsmezo_b200 import AdapterSet
    from step_harness import make_inputs
    mods, bases, *_ = make_inputs(1, 256, 704, 64, 16, 512, 22, torch.bfloat16, torch.bfloat16)
    aset = AdapterSet(mods, bases, 16, 16, copy_dtype=torch.bfloat16, act_dtype=torch.bfloat16, device=DEV)
    T, D = aset.H(0).shape
    with pytest.raises(ValueError):
        aset.load_activations(0, torch.zeros(T + 1, D, device=DEV))
    with pytest.raises(ValueError):
        aset.load_activations(0, torch.zeros(T, D + 1, device=DEV))
    with pytest.raises(TypeError):
        aset.load_activations(0, torch.zeros(T, D, dtype=torch.float16, device=DEV))


@pytest.mark.parametrize("fdt", [torch.bfloat16, torch.float32])
def test_adapter_export_views(fdt):
    # ds_mezo/backend.py:21-36: lora_A.weight = B, lora_B.weight = A, bf16, one per module
    from dsmezo_b200 import ShardedStep
    gen = torch.Generator(device=DEV).manual_seed(9)
    st = ShardedStep(2, 64, 160, 16, 8, 32, eps=1e-3, total_steps=100, generator=gen, copy_dtype=fdt,
                     act_dtype=torch.bfloat16, device=DEV)
    a = st.aset
    g = torch.Generator().manual_seed(1)
    for i in range(len(a.modules)):
        a.A(i).copy_(torch.randn(a.A(i).shape, generator=g))
        a.B(i).copy_(torch.randn(a.B(i).shape, generator=g))
    a.sync_shadow()
    for b in range(len(a.bases)):
        a.V(b).copy_(torch.linalg.qr(torch.randn(a.V(b).shape, generator=g))[0])
        a.H(b).copy_(torch.randn(a.H(b).shape, generator=g))
    st.perturb()
    for which, arena in (("pos", a.pos_dir(0)), ("neg", a.neg_dir(0)), ("factors", a.export_factors)):
        ex = st.export_adapters(which)
        torch.cuda.synchronize()
        assert len(ex) == 2 * len(a.modules)
        for i, m in enumerate(a.modules):
            pre = f"base_model.model.model.layers.{m.layer}." + ("self_attn." if m.name[0] in "qkvo" else "mlp.") + m.name
            A, B = ex[pre + ".lora_B.weight"], ex[pre + ".lora_A.weight"]
            assert A.dtype == torch.bfloat16 and B.dtype == torch.bfloat16
            assert same_bits(A, a.A(i, arena).to(torch.bfloat16)) and same_bits(B, a.B(i, arena).to(torch.bfloat16))
            if fdt == torch.bfloat16:                       # no copy: views of the arena itself
                assert A.data_ptr() == a.A(i, arena).data_ptr() and B.data_ptr() == a.B(i, arena).data_ptr()
