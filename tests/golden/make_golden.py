"""Generate the golden fixtures under tests/golden/ (run in a container that has
the reference tree; the fixtures are committed and then read without it).

Two independent sources of truth, both the reference's own code:
  * oracle/_ref: the reference's scalar C++ path (src/text-decoder.cpp,
    src/gguf-model.cpp) compiled unmodified -> bit-exact expectations
    (prefill logits, layer-0 output, cached greedy ids with and without a
    stop id);
  * the reference's PyTorch restatement (benchmarks/check_text_layer0.py
    `_text_layer_reference`, check_text_generate.py `_prefill_logits_loaded`),
    imported from the reference tree -> float32-tolerance expectations.

The weights are the seeded tiny model of qwenasr.cpp_b200/synth.py; the file
records a checksum of them so a change of the generator is caught.

    python tests/golden/make_golden.py [--ref-root PATH-OF-THE-REFERENCE-TREE]
"""
from __future__ import annotations

import argparse
import hashlib
import sys
import tempfile
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
ROOT = HERE.parents[1]
sys.path.insert(0, str(ROOT))

import __graft_entry__ as ge  # noqa: E402
from oracle import oracle as checker  # noqa: E402


def weights_digest(tensors: dict) -> str:
    h = hashlib.sha256()
    for name in sorted(tensors):
        h.update(name.encode())
        h.update(np.ascontiguousarray(tensors[name]).tobytes())
    return h.hexdigest()


def torch_reference(ref_root: Path, cfg: dict, tensors: dict, x: np.ndarray, n_new: int):
    import torch

    sys.path.insert(0, str(ref_root / "benchmarks"))
    import check_text_generate as ctg  # the reference's torch restatement
    import check_text_layer0 as ctl

    names = {"attn_norm_weight": "attn_norm", "ffn_norm_weight": "ffn_norm", "q_weight": "attn_q",
             "k_weight": "attn_k", "v_weight": "attn_v", "out_weight": "attn_output", "q_norm_weight": "attn_q_norm",
             "k_norm_weight": "attn_k_norm", "gate_weight": "ffn_gate", "up_weight": "ffn_up",
             "down_weight": "ffn_down"}
    layers = [{k: torch.from_numpy(np.array(tensors[f"text.blk.{l}.{v}.weight"])) for k, v in names.items()}
              for l in range(cfg["n_layers"])]
    out_norm = torch.from_numpy(np.array(tensors["text.output_norm.weight"]))
    out_w = torch.from_numpy(np.array(tensors["text.output.weight"]))
    embd = torch.from_numpy(np.array(tensors["text.token_embd.weight"]))
    text_cfg = {"num_attention_heads": cfg["n_heads"], "num_key_value_heads": cfg["n_kv_heads"],
                "head_dim": cfg["head_dim"], "rope_theta": cfg["rope_theta"], "rms_norm_eps": cfg["rms_norm_eps"]}
    xt = torch.from_numpy(x.copy())
    with torch.no_grad():
        layer0 = ctl._text_layer_reference(xt, layers[0], heads=cfg["n_heads"], kv_heads=cfg["n_kv_heads"],
                                           head_dim=cfg["head_dim"], rope_theta=cfg["rope_theta"],
                                           eps=cfg["rms_norm_eps"]).numpy()
        logits = ctg._prefill_logits_loaded(xt, layers, out_norm, out_w, text_cfg).numpy()
        ids = []
        cur = xt
        for _ in range(n_new):   # the recompute greedy loop of check_text_generate.py:_torch_generate
            lg = ctg._prefill_logits_loaded(cur, layers, out_norm, out_w, text_cfg)
            nid = int(lg.argmax().item())
            ids.append(nid)
            cur = torch.cat([cur, embd[nid].view(1, -1)], dim=0)
    return layer0.astype(np.float32), logits.astype(np.float32), np.asarray(ids, np.int32)


def main() -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref-root", type=Path, default=HERE.parents[2] / "reference",
                    help="reference checkout (default: beside this repository)")
    ap.add_argument("--out", type=Path, default=HERE)
    a = ap.parse_args()
    synth = ge.load_synth()
    checker.build(ref=True)
    cfg = dict(synth.TINY)
    n_new = 16
    with tempfile.TemporaryDirectory() as td:
        for norm in ("normal", "one_plus"):
            path = synth.write_gguf(Path(td) / f"tiny_{norm}.gguf", cfg, seed=0, norm_init=norm)
            tensors = synth.read_gguf(path)
            rng = np.random.default_rng(20)
            x, _ = synth.prompt_rows(tensors["text.token_embd.weight"], 24, rng, audio_rows=14, audio_start=3)
            ref = checker.RefModel(path, cfg)
            logits = ref.prefill_logits(x)
            layer0 = ref.layer_forward(0, x)
            ids, stopped = ref.generate_cached(x, n_new)
            stop_id = int(ids[5])
            ids_stop, stopped_stop = ref.generate_cached(x, n_new, stop_ids=[stop_id])
            t_layer0, t_logits, t_ids = torch_reference(a.ref_root, cfg, tensors, x, 8)
            np.savez_compressed(
                a.out / f"tiny_{norm}.npz", x=x, weights_sha256=np.array(weights_digest(tensors)),
                ref_prefill_logits=logits, ref_layer0=layer0, ref_ids=ids, ref_stopped=np.array(stopped),
                stop_id=np.array(stop_id), ref_ids_stop=ids_stop, ref_stopped_stop=np.array(stopped_stop),
                torch_layer0=t_layer0, torch_prefill_logits=t_logits, torch_ids=t_ids)
            print(f"{norm}: ids={ids.tolist()} stop@{stop_id}->{ids_stop.tolist()} torch_ids={t_ids.tolist()}")
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
