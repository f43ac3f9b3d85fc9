"""CPU stand-ins for the single-GPU kernel stages, built from the oracle.

Used only by the gloo tests of the expert-parallel host logic (planning,
count exchange, all-to-all of rows, tile tables), which need no GPU.
"""
import numpy as np
import torch
import torch.nn.functional as F

from oracle import permute_oracle


class OracleLocalOps:
    def route(self, x, w_router, top_k):
        E = w_router.shape[0]
        logits = F.linear(x, w_router).float()
        vals, idx = torch.topk(logits, top_k, dim=-1)
        gates = vals.softmax(-1).to(x.dtype)
        counts, seg, row_of, token_of, _ = permute_oracle.dispatch_layout_fast(idx.numpy(), E)
        x_perm = torch.zeros(int(seg[-1]), x.shape[1], dtype=x.dtype)
        tok = torch.from_numpy(token_of)
        x_perm[tok >= 0] = x[tok[tok >= 0]]
        return idx, gates, x_perm, torch.from_numpy(row_of), torch.from_numpy(counts.astype(np.int32))

    def ffn(self, rows, w1, b1, w2, b2, tile_expert):
        out = torch.empty(rows.shape[0], w2.shape[1], dtype=rows.dtype)
        for m, e in enumerate(tile_expert.tolist()):
            r = rows[m * 128:(m + 1) * 128]
            out[m * 128:(m + 1) * 128] = F.linear(torch.relu(F.linear(r, w1[e], b1[e])), w2[e], b2[e])
        return out

    def combine(self, y_perm, row_of, gates):
        out = torch.zeros(row_of.shape[0], y_perm.shape[1], dtype=y_perm.dtype)
        ar = torch.arange(row_of.shape[0])
        for r in range(row_of.shape[1]):
            out.index_add_(0, ar, y_perm[row_of[:, r].long()] * gates[:, r:r + 1])
        return out
