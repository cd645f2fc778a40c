"""Helpers that turn a golden fixture ([M,B,T,H,d] reference layout) into flat streams."""
import glob
import os

import numpy as np

GOLDEN_DIR = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def golden_files():
    """Attention fixtures (the reference's BatchedACE modules)."""
    return sorted(p for p in glob.glob(os.path.join(GOLDEN_DIR, "*.npz"))
                  if not os.path.basename(p).startswith(("probs_", "g_", "mod_")))


def module_files():
    """Module fixtures (the reference's RACEAttention / RACEBlock, both files)."""
    return sorted(glob.glob(os.path.join(GOLDEN_DIR, "mod_*.npz")))


def load_module(path):
    """(meta dict, state_dict of float32 tensors, fixture arrays) of a module fixture."""
    import json

    import torch
    z = np.load(path)
    meta = json.loads(str(z["meta_json"]))
    sd = {k[3:]: torch.tensor(z[k]) for k in z.files if k.startswith("sd/")}
    return meta, sd, {k: z[k] for k in z.files}


def build_module(meta, device="cpu"):
    """The drop-in module matching a fixture's reference class and arguments."""
    from race_attention_b200 import race as R, vit as V
    mod = V if meta["file"] == "misc/vit.py" else R
    skip = {"file", "cls", "kind", "B", "T", "d_model"}
    args = {k: v for k, v in meta.items() if k not in skip}
    if meta["kind"] == "block":
        return mod.RACEBlock(args, device=device)
    return mod.RACEAttention(**args, device=device)


def probs_files():
    """Probability-export fixtures (the reference's race_bucket_probs_from_qk)."""
    return sorted(glob.glob(os.path.join(GOLDEN_DIR, "probs_*.npz")))


def global_files():
    """Global-normalisation fixtures (the reference's CausalRACEAttention)."""
    return sorted(glob.glob(os.path.join(GOLDEN_DIR, "g_*.npz")))


def load_global(path):
    """A CausalRACEAttention fixture as flat streams.

    q, k, v, dout: [B, T, H*dk] -> [B*H, T, dk]; the mask (if any) is applied to
    k and v as the reference does before hashing; planes [L, K, dk] ->
    [B*H, L*K, dk]; dden: the gradient the fixture's d_token loss puts on the
    per-stream, table-summed denominator (d_token = mean_h(den) / L), zero
    where d_token's clamp holds."""
    z = np.load(path)
    B, T, H, dk, K, L, C, masked = [int(x) for x in z["meta"]]
    g = {k: z[k] for k in z.files}
    split = lambda x: np.ascontiguousarray(
        x.reshape(B, T, H, dk).transpose(0, 2, 1, 3).reshape(B * H, T, dk))
    keep = g["mask"] if masked else np.ones((B, T), np.float32)
    keep_s = np.repeat(keep, H, axis=0)[:, :, None]                   # [B*H, T, 1]
    gtok = g["gtok"][..., 0]                                           # [B, T]
    live = g["d_token"][..., 0] >= 1e-6
    dden = np.repeat(np.where(live, gtok, 0.0) / (H * L), H, axis=0)
    g.update(B=B, T=T, H=H, hd=dk, K=K, L=L, C=C, masked=bool(masked),
             name=os.path.basename(path)[:-4], split=split, keep_s=keep_s, dden=dden,
             qs=split(g["q"]), ks=split(g["k"]) * keep_s, vs=split(g["v"]) * keep_s,
             douts=split(g["dout"]),
             planes_s=np.broadcast_to(g["planes"].reshape(1, L * K, dk), (B * H, L * K, dk)))
    return g


def merge_heads(xs, B, H):
    """[B*H, T, dk] -> [B, T, H*dk]."""
    N, T, dk = xs.shape
    return xs.reshape(B, H, T, dk).transpose(0, 2, 1, 3).reshape(B, T, H * dk)


def load(path):
    z = np.load(path)
    M, B, T, H, d, K, L, share, causal = [int(x) for x in z["meta"]]
    g = {k: z[k] for k in z.files}
    g.update(M=M, B=B, T=T, H=H, d=d, K=K, L=L, share=bool(share), causal=bool(causal),
             name=os.path.basename(path)[:-4])
    return g


def to_streams(x5):
    """[M,B,T,H,d] -> [M*B*H, T, d] in (m, b, h) stream order."""
    M, B, T, H, d = x5.shape
    return np.ascontiguousarray(x5.transpose(0, 1, 3, 2, 4).reshape(M * B * H, T, d))


def from_streams(xs, M, B, H):
    N, T, d = xs.shape
    return xs.reshape(M, B, H, T, d).transpose(0, 1, 3, 2, 4)


def stream_planes(g):
    """planes per stream: [M*B*H, L*K, d]."""
    P = g["planes"]                      # [Mp, LK, d]
    M, B, H = g["M"], g["B"], g["H"]
    idx = np.repeat(np.arange(M) if P.shape[0] == M else np.zeros(M, int), B * H)
    return P[idx]


def inputs_as_streams(g):
    """q,k,v [B,T,H,d] shared by all ensembles (the reference expands them)."""
    M = g["M"]
    ex = lambda x: np.broadcast_to(x[None], (M,) + x.shape)
    return to_streams(ex(g["q"])), to_streams(ex(g["k"])), to_streams(ex(g["v"]))
