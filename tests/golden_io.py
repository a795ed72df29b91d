"""Loading helpers for the committed golden vectors (tests/golden/*.npz)."""
import glob
import os

import numpy as np

GOLDEN_DIR = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def golden_names():
    return sorted(os.path.splitext(os.path.basename(p))[0]
                  for p in glob.glob(os.path.join(GOLDEN_DIR, "*.npz")))


def load_golden(name):
    z = np.load(os.path.join(GOLDEN_DIR, f"{name}.npz"))
    d = {k: z[k] for k in z.files}
    d["q_f32"] = (d["q_bf16"].astype(np.uint32) << 16).view(np.float32)
    d["out_f32"] = (d["out_bf16"].astype(np.uint32) << 16).view(np.float32)
    d["topk_length"] = d["topk_length"] if bool(d["has_topk_length"]) else None
    d["attn_sink"] = d["attn_sink"] if bool(d["has_sink"]) else None
    d["sm_scale"] = float(d["sm_scale"])
    d["page_block"] = int(d["page_block"])
    return d
