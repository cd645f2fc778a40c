"""Helpers that turn a golden fixture ([M,B,T,H,d] reference layout) into flat streams."""
import glob
import os

import numpy as np

GOLDEN_DIR = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def golden_files():
    """Attention fixtures (the reference's BatchedACE modules)."""
    return sorted(p for p in glob.glob(os.path.join(GOLDEN_DIR, "*.npz"))
                  if not os.path.basename(p).startswith("probs_"))


def probs_files():
    """Probability-export fixtures (the reference's race_bucket_probs_from_qk)."""
    return sorted(glob.glob(os.path.join(GOLDEN_DIR, "probs_*.npz")))


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
