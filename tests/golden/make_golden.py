"""Generate golden vectors from the reference implementation itself.

Runs DS-MeZO's own code on CPU and records inputs and outputs:

* ``ds_mezo/kernels.py`` (all four Triton kernels) under ``TRITON_INTERPRET=1``;
* ``ds_mezo/controller.py`` ``DSMeZO_Controller`` (constructor, ``_perturb_and_sync``,
  ``_update_weights``, ``_step_lr``), with stand-ins only for what cannot run here:
  the vLLM backend (no rollout), ``peft``/``optht`` (not installed, unused on this path),
  ``safetensors.load_file`` (returns the in-memory adapter), and ``device="cuda"``
  (mapped to CPU). The CUDA generator is replaced by a CPU generator whose draws are
  recorded, so the fixtures carry the exact Gaussian values the reference consumed.
* ``ds_mezo/controller.py`` ``_score_contrastive`` (with ``_mean_nll``) on a stub backend
  that returns the fp32 log-softmax logprobs of seeded logits (``scoring.pt``).

Usage (needs the reference checkout; writes tests/golden/*.pt):
    python tests/golden/make_golden.py --ref <reference checkout>   (or DSMEZO_REFERENCE=<path>)
"""
from __future__ import annotations

import argparse
import importlib.util
import os
import sys
import types
from pathlib import Path

os.environ["TRITON_INTERPRET"] = "1"
import torch  # noqa: E402

HERE = Path(__file__).resolve().parent


class _TorchProxy(types.ModuleType):
    """Forwards to torch but maps device='cuda' to CPU and records randn draws."""

    def __init__(self, recorder):
        super().__init__("torch")
        self._rec = recorder

    def __getattr__(self, name):
        return getattr(torch, name)

    def empty(self, *a, device=None, **k):
        return torch.empty(*a, **k)

    def zeros(self, *a, device=None, **k):
        return torch.zeros(*a, **k)

    def Generator(self, device=None):  # noqa: N802
        return torch.Generator()

    def randn(self, *shape, device=None, generator=None, **k):
        t = torch.randn(*shape, generator=generator, **k)
        self._rec.append(t.clone())
        return t


def load_reference(ref: Path, recorder):
    peft = types.ModuleType("peft")
    peft.PeftConfig = object
    peft.LoraConfig = object
    optht = types.ModuleType("optht")
    optht.optht = lambda *a, **k: 0
    sys.modules.setdefault("peft", peft)
    sys.modules.setdefault("optht", optht)

    pkg = types.ModuleType("ds_mezo")
    pkg.__path__ = [str(ref / "ds_mezo")]
    sys.modules["ds_mezo"] = pkg

    def load(name, path):
        spec = importlib.util.spec_from_file_location(name, path)
        mod = importlib.util.module_from_spec(spec)
        sys.modules[name] = mod
        spec.loader.exec_module(mod)
        return mod

    kernels = load("ds_mezo.kernels", ref / "ds_mezo" / "kernels.py")
    kernels.torch = _TorchProxy(recorder)
    backend = types.ModuleType("ds_mezo.backend")
    backend.save_peft_adapter = lambda *a, **k: None
    backend.write_adapter_config = lambda *a, **k: None
    sys.modules["ds_mezo.backend"] = backend
    model_config = load("ds_mezo.model_config", ref / "ds_mezo" / "model_config.py")
    controller = load("ds_mezo.controller", ref / "ds_mezo" / "controller.py")
    controller.torch = _TorchProxy(recorder)
    return kernels, controller, model_config


def kernel_cases(K, g):
    """Per-kernel fixtures on small and odd shapes the Triton kernels accept."""
    floor = float(torch.finfo(torch.float32).tiny)
    out = {"ns_c1": torch.tensor(K._NS_C1, dtype=torch.float64),
           "ns_c3": torch.tensor(K._NS_C3, dtype=torch.float64)}
    # zo_muon: tall needs pow2 N, wide needs pow2 M (tl.arange over the short side)
    for name, (M, N) in {"tall_1408x8": (1408, 8), "tall_200x16": (200, 16), "tall_16x16": (16, 16),
                         "wide_8x512": (8, 512), "wide_16x1000": (16, 1000), "wide_4x37": (4, 37)}.items():
        param = torch.randn(M, N, generator=g)
        buf = torch.randn(M, N, generator=g)
        scratch = torch.zeros(M, N)
        p0 = param.clone()
        K.zo_muon_update(param, buf, scratch, 0.01, floor)
        out[f"muon_{name}"] = {"param_in": p0, "buf": buf, "eta": 0.01, "param_out": param.clone(),
                                "scratch_out": scratch.clone()}
    # power iteration (D, R padded to pow2 inside the kernel)
    for name, (T, D, R) in {"t256_d512_r8": (256, 512, 8), "t64_d200_r8": (64, 200, 8),
                            "t130_d96_r16": (130, 96, 16), "t32_d48_r5": (32, 48, 5)}.items():
        scale = torch.exp(torch.randn(D, generator=g))
        H = torch.randn(T, D, generator=g) * scale
        V0 = torch.linalg.qr(torch.randn(D, R, generator=g))[0].contiguous()
        V = K.fused_power_iter(H, V0, num_iters=3, norm_floor=floor)
        out[f"pi_{name}"] = {"H": H, "V0": V0, "iters": 3, "V": V.clone()}
    # AGZO perturbation (R, RC pow2 inside the kernel)
    for name, (d_out, R, d_in, RC) in {"q_128x8x512_rc8": (128, 8, 512, 8), "o_300x8x200_rc4": (300, 8, 200, 4),
                                        "k_64x4x96_rc8": (64, 4, 96, 8), "g_704x16x256_rc16": (704, 16, 256, 16)}.items():
        B = torch.randn(R, d_in, generator=g)
        V = torch.linalg.qr(torch.randn(d_in, RC, generator=g))[0].contiguous()
        zcB = torch.randn(R, RC, generator=g).contiguous()
        zcA = torch.randn(d_out, min(R, RC), generator=g).contiguous()
        z_A, z_B = K.fused_agzo_perturbation(B, V, zcB, zcA, 1e-3, floor)
        out[f"agzo_{name}"] = {"B": B, "V": V, "zcB": zcB, "zcA": zcA, "eps": 1e-3,
                               "z_A": z_A.clone(), "z_B": z_B.clone()}
    base = torch.randn(1000, generator=g)
    z = torch.randn(1000, generator=g) * 1e-3
    pos, neg = torch.empty(1000), torch.empty(1000)
    K.fused_perturb_dual(base, z, pos, neg)
    out["dual"] = {"base": base, "z": z, "pos": pos, "neg": neg}
    return out


class _Cfg:
    def __init__(self, total_steps, seed, out_dir, adapter_path):
        self.output_dir = out_dir
        self.training = types.SimpleNamespace(total_steps=total_steps, seed=seed, resume_from="")
        self.model = types.SimpleNamespace(adapter_path=adapter_path)


def controller_case(C, MC, g, *, layers, h, inter, kv, r, T, steps, total_steps, seed, tmp):
    """Runs the reference controller for ``steps`` optimizer steps on a synthetic set."""
    shapes = {"q_proj": (h, h), "k_proj": (kv, h), "v_proj": (kv, h), "o_proj": (h, h),
              "gate_proj": (inter, h), "up_proj": (inter, h), "down_proj": (h, inter)}
    specs, tensors = [], {}
    for li in range(layers):
        for mod in sorted(shapes):
            d_out, d_in = shapes[mod]
            prefix = f"base_model.model.model.layers.{li}.mlp.{mod}"
            specs.append(MC.LayerSpec(layer_idx=li, module_name=mod, peft_prefix=prefix))
            tensors[f"{prefix}.lora_A.weight"] = torch.randn(r, d_in, generator=g)   # = B
            tensors[f"{prefix}.lora_B.weight"] = torch.randn(d_out, r, generator=g)  # = A
    specs.sort(key=lambda s: (s.layer_idx, s.module_name))
    C.load_file = lambda path, device=None: {k: v.clone() for k, v in tensors.items()}

    class _Backend:
        def sync_adapters(self, *a, **k):
            pass

    cfg = _Cfg(total_steps, seed, str(tmp), str(tmp))
    ctrl = C.DSMeZO_Controller(_Backend(), specs, cfg, score_fn=None)
    rec = C.torch._rec
    rec.clear()

    def snapshot():
        return {f"{l.layer_idx}.{l.module_name}": {
            "A": l.A.clone(), "B": l.B.clone(), "mu_A": l.momentum_A.clone(), "mu_B": l.momentum_B.clone(),
            "var_A": l.variance_A.clone(), "var_B": l.variance_B.clone()} for l in ctrl.layers}

    # one unique activation per (layer, input): qkv share, gate/up share (ds_mezo/backend.py:49-52)
    groups = {"qkv": ("q_proj", "k_proj", "v_proj"), "o": ("o_proj",), "gu": ("gate_proj", "up_proj"),
              "down": ("down_proj",)}
    in_dim = {"qkv": h, "o": h, "gu": h, "down": inter}
    ctrl.r_calib = r
    record = {"config": dict(layers=layers, h=h, inter=inter, kv=kv, r=r, T=T, total_steps=total_steps,
                             seed=seed, eps=ctrl.eps, eta_max=ctrl.eta_max, eta_min=ctrl.eta_min,
                             power_iter_steps=ctrl.power_iter_steps),
              "init": snapshot(), "steps": []}
    bases = {}
    for li in range(layers):
        for gname, mods in groups.items():
            V0 = torch.linalg.qr(torch.randn(in_dim[gname], r, generator=g))[0].contiguous()
            for mod in mods:
                ctrl.activation_bases[(li, mod)] = V0
            bases[f"{li}.{gname}"] = V0.clone()
    record["bases0"] = bases
    orig_cuda = torch.Tensor.cuda
    torch.Tensor.cuda = lambda self, *a, **k: self
    try:
        for s in range(steps):
            acts, act_rec = {}, {}
            for li in range(layers):
                for gname, mods in groups.items():
                    scale = torch.exp(torch.randn(in_dim[gname], generator=g))
                    Hm = torch.randn(T, in_dim[gname], generator=g) * scale
                    act_rec[f"{li}.{gname}"] = Hm.clone()
                    for mod in mods:
                        acts[(li, mod)] = Hm
            ctrl.step_count += 1
            rec.clear()
            perts = ctrl._perturb_and_sync(acts)
            draws = [t.clone() for t in rec]
            dd = float(torch.randn((), generator=g)) * 10.0
            eta_used = ctrl.eta
            ctrl._update_weights(perts, dd)
            step = {"activations": act_rec, "draws": draws, "dd": dd, "eta": eta_used,
                    "eta_after": ctrl.eta, "step_count": ctrl.step_count,
                    "z": {f"{l.layer_idx}.{l.module_name}": (perts[l.key][0].clone(), perts[l.key][1].clone())
                          for l in ctrl.layers},
                    "pos": {f"{l.layer_idx}.{l.module_name}": (l.pos_A.clone(), l.pos_B.clone()) for l in ctrl.layers},
                    "neg": {f"{l.layer_idx}.{l.module_name}": (l.neg_A.clone(), l.neg_B.clone()) for l in ctrl.layers},
                    "bases": {f"{li}.{gname}": ctrl.activation_bases[(li, groups[gname][0])].clone()
                              for li in range(layers) for gname in groups},
                    "state": snapshot()}
            record["steps"].append(step)
    finally:
        torch.Tensor.cuda = orig_cuda
    return record


def scoring_cases(C, g):
    """ds_mezo/controller.py:194-201 (_score_contrastive, with _mean_nll at :14-15) on a stub
    backend whose score() returns, per trajectory, the fp32 log-softmax logprob of each
    token after the first (what ds_mezo/backend.py:98-103 extracts from vLLM). Records the
    scored rows' logits and targets so that the device reduction can start from logits."""
    cases = []
    for n_traj, prompt_len, vocab, max_new in [(4, 5, 50, 9), (4, 12, 256, 30), (2, 3, 1000, 4), (6, 1, 17, 6)]:
        lens = [prompt_len + int(torch.randint(1, max_new + 1, (1,), generator=g)) for _ in range(n_traj)]
        trajs = [torch.randint(0, vocab, (L,), generator=g).tolist() for L in lens]
        adv = (torch.randn(n_traj, generator=g) * 0.7).tolist()
        logits = {k: [torch.randn(L - 1, vocab, generator=g) * 3 for L in lens] for k in ("pos", "neg")}

        class _Score:
            lora_pos, lora_neg = "pos", "neg"

            def score(self, trajectories, lora):
                out = []
                for t, lg in zip(trajectories, logits[lora]):
                    lp = torch.log_softmax(lg, dim=-1)
                    out.append([float(lp[j, t[j + 1]]) for j in range(len(t) - 1)])
                return out

        fake = types.SimpleNamespace(backend=_Score())
        loss_pos, loss_neg = C.DSMeZO_Controller._score_contrastive(fake, trajs, adv, prompt_len)
        rows = {k: torch.cat([lg[prompt_len - 1:] for lg in logits[k]]) for k in ("pos", "neg")}
        targets = torch.tensor([tok for t in trajs for tok in t[prompt_len:]], dtype=torch.int32)
        cases.append({"prompt_len": prompt_len, "lens": lens, "advantages": adv, "seq_tokens": [L - prompt_len for L in lens],
                      "targets": targets, "rows_pos": rows["pos"], "rows_neg": rows["neg"],
                      "loss_pos": float(loss_pos), "loss_neg": float(loss_neg)})
    return cases


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref", default=os.environ.get("DSMEZO_REFERENCE"),
                    help="path of the reference checkout (default: $DSMEZO_REFERENCE)")
    ap.add_argument("--only", choices=["scoring"], default=None, help="write only this fixture")
    args = ap.parse_args()
    if not args.ref:
        ap.error("give the reference checkout with --ref or DSMEZO_REFERENCE")
    rec = []
    K, C, MC = load_reference(Path(args.ref), rec)
    torch.save(scoring_cases(C, torch.Generator().manual_seed(31)), HERE / "scoring.pt")
    if args.only == "scoring":
        print("wrote scoring.pt")
        return
    g = torch.Generator().manual_seed(20260)
    torch.save(kernel_cases(K, g), HERE / "kernels.pt")
    import tempfile
    with tempfile.TemporaryDirectory() as tmp:
        g = torch.Generator().manual_seed(7)
        mini = controller_case(C, MC, g, layers=2, h=64, inter=176, kv=16, r=8, T=48, steps=2,
                               total_steps=100, seed=0, tmp=tmp)
        torch.save(mini, HERE / "controller_mini.pt")
    print("wrote", sorted(p.name for p in HERE.glob("*.pt")))


if __name__ == "__main__":
    main()
