"""Times the reference's own optimizer step on CPU: ``ds_mezo/kernels.py`` under
``TRITON_INTERPRET=1`` driven by ``DSMeZO_Controller._perturb_and_sync`` and
``_update_weights`` (ds_mezo/controller.py:236-292; the power iteration, perturbation, dual
copies, Kalman update and ZO-Muon of every module), with the stand-ins of
``tests/golden/make_golden.py`` for what cannot run on a CPU (vLLM backend, CUDA device
and generator).

Test infrastructure: it needs the reference checkout (``--ref`` or ``DSMEZO_REFERENCE``),
so it runs only where that checkout is, never on a GPU host. It prints one JSON line per
config with the seconds per step and the host threads torch used.

    python oracle/interpreted_reference.py --ref <reference checkout> --config toy [--steps 1]
"""
from __future__ import annotations

import argparse
import importlib.util
import json
import os
import tempfile
import time
from pathlib import Path

os.environ["TRITON_INTERPRET"] = "1"
import torch  # noqa: E402

ROOT = Path(__file__).resolve().parents[1]
SHAPES = {   # layers, hidden, intermediate, kv_out, rank, tokens (the bench's configs)
    "toy": (4, 512, 1408, 128, 8, 256),
    "1.5b": (28, 1536, 8960, 256, 16, 2048),
}


def _golden_module():
    spec = importlib.util.spec_from_file_location("make_golden", ROOT / "tests" / "golden" / "make_golden.py")
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def time_step(ref: Path, config: str, steps: int, layers: int = 0):
    mg = _golden_module()
    rec = []
    K, C, MC = mg.load_reference(ref, rec)
    L, h, inter, kv, r, T = SHAPES[config]
    if layers:
        L = layers
    g = torch.Generator().manual_seed(0)
    shapes = {"q_proj": (h, h), "k_proj": (kv, h), "v_proj": (kv, h), "o_proj": (h, h),
              "gate_proj": (inter, h), "up_proj": (inter, h), "down_proj": (h, inter)}
    specs, tensors = [], {}
    for li in range(L):
        for mod in sorted(shapes):
            d_out, d_in = shapes[mod]
            prefix = f"base_model.model.model.layers.{li}.mlp.{mod}"
            specs.append(MC.LayerSpec(layer_idx=li, module_name=mod, peft_prefix=prefix))
            tensors[f"{prefix}.lora_A.weight"] = torch.randn(r, d_in, generator=g)
            tensors[f"{prefix}.lora_B.weight"] = torch.randn(d_out, r, generator=g)
    specs.sort(key=lambda s: (s.layer_idx, s.module_name))
    C.load_file = lambda path, device=None: {k: v.clone() for k, v in tensors.items()}

    class _Backend:
        def sync_adapters(self, *a, **k):
            pass

    groups = {"qkv": ("q_proj", "k_proj", "v_proj"), "o": ("o_proj",), "gu": ("gate_proj", "up_proj"),
              "down": ("down_proj",)}
    in_dim = {"qkv": h, "o": h, "gu": h, "down": inter}
    with tempfile.TemporaryDirectory() as tmp:
        ctrl = C.DSMeZO_Controller(_Backend(), specs, mg._Cfg(1000, 0, tmp, tmp), score_fn=None)
        ctrl.r_calib = r
        acts = {}
        for li in range(L):
            for gname, mods in groups.items():
                V0 = torch.linalg.qr(torch.randn(in_dim[gname], r, generator=g))[0].contiguous()
                Hm = torch.randn(T, in_dim[gname], generator=g) * torch.exp(torch.randn(in_dim[gname], generator=g))
                for mod in mods:
                    ctrl.activation_bases[(li, mod)] = V0
                    acts[(li, mod)] = Hm
        orig_cuda = torch.Tensor.cuda
        torch.Tensor.cuda = lambda self, *a, **k: self
        try:
            times = []
            for _ in range(steps):
                ctrl.step_count += 1
                t0 = time.perf_counter()
                perts = ctrl._perturb_and_sync(acts)
                ctrl._update_weights(perts, 1.0)
                times.append(time.perf_counter() - t0)
        finally:
            torch.Tensor.cuda = orig_cuda
    return {"config": config, "layers": L, "seconds_per_step": sum(times) / len(times), "steps": steps,
            "threads": torch.get_num_threads(), "cpu_count": os.cpu_count(),
            "what": "ds_mezo/kernels.py under TRITON_INTERPRET=1 + DSMeZO_Controller._perturb_and_sync/_update_weights"}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref", default=os.environ.get("DSMEZO_REFERENCE"))
    ap.add_argument("--config", choices=sorted(SHAPES), default="toy")
    ap.add_argument("--steps", type=int, default=1)
    ap.add_argument("--layers", type=int, default=0, help="time the first N layers only (0: all)")
    a = ap.parse_args()
    if not a.ref:
        ap.error("give the reference checkout with --ref or DSMEZO_REFERENCE")
    print(json.dumps(time_step(Path(a.ref), a.config, a.steps, a.layers)), flush=True)


if __name__ == "__main__":
    main()
