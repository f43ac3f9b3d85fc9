"""Loading helpers for the golden vectors in tests/golden/*.npz."""
import glob
import hashlib
import os

import numpy as np
import torch

from oracle.golden_cases import case_by_name, case_inputs

GOLDEN_DIR = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
DTYPES = {"float32": torch.float32, "bfloat16": torch.bfloat16, "float16": torch.float16}


def _all_names():
    return sorted(os.path.basename(p)[:-4] for p in glob.glob(os.path.join(GOLDEN_DIR, "*.npz")))


def names():
    """Forward (and gradient) cases of the MoE block."""
    return [n for n in _all_names() if not n.startswith(("aux_", "codec_"))]


def aux_names():
    """Auxiliary-loss cases (tests/golden/make_golden_aux.py)."""
    return [n for n in _all_names() if n.startswith("aux_")]


def _to_np(t):
    t = t.detach().cpu().contiguous()
    if t.dtype == torch.bfloat16:
        return t.view(torch.int16).numpy().view(np.uint16)
    return t.numpy()


def sha(t):
    return hashlib.sha256(_to_np(t).tobytes()).hexdigest()


def state_sha(sd):
    h = hashlib.sha256()
    for k in sorted(sd):
        h.update(k.encode())
        h.update(_to_np(sd[k]).tobytes())
    return h.hexdigest()


def from_np(a, dtype):
    if dtype == torch.bfloat16:
        return torch.from_numpy(np.ascontiguousarray(a).view(np.int16)).view(torch.bfloat16)
    return torch.from_numpy(np.ascontiguousarray(a))


class Golden:
    """One golden case: regenerated inputs (hash-checked) and reference outputs."""

    def __init__(self, name):
        self.name = name
        self.z = np.load(os.path.join(GOLDEN_DIR, name + ".npz"))
        z = self.z
        self.case = case_by_name(name)
        self.dtype = DTYPES[str(z["dtype"])]
        self.top_k = int(z["top_k"])
        self.E = int(z["experts"])
        self.d = int(z["d"])
        self.H = int(z["hidden"])
        self.N = int(z["n_tokens"])
        self.shared = int(z["shared"])
        sd32, x32 = case_inputs(self.case)
        self.sd = {k: v.to(self.dtype) for k, v in sd32.items()}
        self.x = x32.to(self.dtype)
        self.out = from_np(z["out"], self.dtype)
        self.logits = torch.from_numpy(z["logits"])
        self.idx = torch.from_numpy(z["idx"].astype(np.int64))
        self.gates = from_np(z["gates"], self.dtype)
        self.counts = torch.from_numpy(z["counts"].astype(np.int64))

    def inputs_match(self):
        return sha(self.x) == str(self.z["x_sha256"]) and state_sha(self.sd) == str(self.z["state_sha256"])


def grad_names():
    return sorted(n for n in names() if n.startswith("grad_"))


class GoldenGrad(Golden):
    """A gradient case: the reference's backward (tests/golden/make_golden_grads.py)."""

    def __init__(self, name):
        super().__init__(name)
        from oracle.golden_cases import grad_output

        z = self.z
        self.dout = grad_output(self.case).to(self.dtype)
        self.dx = from_np(z["dx"], self.dtype)
        self.d_router = from_np(z["d_router"], self.dtype)
        self.d_w1 = from_np(z["d_w1"], self.dtype)
        self.d_b1 = from_np(z["d_b1"], self.dtype)
        self.d_w2 = from_np(z["d_w2"], self.dtype)
        self.d_b2 = from_np(z["d_b2"], self.dtype)
        self.expert_has_grad = [bool(v) for v in z["expert_has_grad"]]
        self.shared_grads = {}
        if self.shared:
            for i, a, p in ((0, "w1", "weight"), (0, "b1", "bias"), (2, "w2", "weight"), (2, "b2", "bias")):
                stack = from_np(z[f"d_s{i}{a}"], self.dtype)
                for s in range(self.shared):
                    self.shared_grads[f"shared.{s}.{i}.{p}"] = stack[s]

    def inputs_match(self):
        return super().inputs_match() and sha(self.dout) == str(self.z["dout_sha256"])

    def grads(self):
        """Reference gradients keyed like the state dict (zeros for experts
        without a gradient)."""
        g = {"router.weight": self.d_router}
        for e in range(self.E):
            g[f"experts.{e}.0.weight"] = self.d_w1[e]
            g[f"experts.{e}.0.bias"] = self.d_b1[e]
            g[f"experts.{e}.2.weight"] = self.d_w2[e]
            g[f"experts.{e}.2.bias"] = self.d_b2[e]
        g.update(self.shared_grads)
        return g


class GoldenAux:
    """An auxiliary-loss case: per module the stashed router input and router
    weight (as stored, and as regenerated from the seeds), the reference's
    loss and its router weight gradients for the stored upstream gradient."""

    def __init__(self, name):
        from oracle.golden_cases import aux_case_inputs

        self.name = name
        z = self.z = np.load(os.path.join(GOLDEN_DIR, name + ".npz"))
        self.case = case_by_name(name)
        self.dtype = DTYPES[str(z["dtype"])]
        self.E = int(z["experts"])
        self.d = int(z["d"])
        self.N = int(z["n_tokens"])
        self.aux_coef = float(z["aux_coef"])
        self.z_coef = float(z["z_coef"])
        self.upstream = float(z["upstream"])
        self.modules = int(z["modules"])
        self.xs = [from_np(z[f"x{i}"], self.dtype) for i in range(self.modules)]
        self.ws = [from_np(z[f"w{i}"], self.dtype) for i in range(self.modules)]
        self.d_router = [from_np(z[f"d_router{i}"], self.dtype) for i in range(self.modules)]
        self.loss = torch.tensor(float(z["loss"]), dtype=torch.float32)
        self.regenerated = [(x.to(self.dtype), w.to(self.dtype)) for x, w in aux_case_inputs(self.case)]

    def inputs_match(self):
        return all(torch.equal(x, xr) and torch.equal(w, wr)
                   for x, w, (xr, wr) in zip(self.xs, self.ws, self.regenerated))


def codec_names():
    """Tensor-codec cases (tests/golden/make_golden_codec.py)."""
    return [n for n in _all_names() if n.startswith("codec_")]


class GoldenCodec:
    """A tensor-codec case: the reference's encoded state for one encoder
    mode (rebuilt from the stored metadata and payload bytes), its decoded
    values and the targets after each side-update application."""

    def __init__(self, name):
        import json

        self.name = name
        z = self.z = np.load(os.path.join(GOLDEN_DIR, name + ".npz"))
        self.mode = str(z["mode"])
        self.meta = json.loads(str(z["meta"]))
        header = json.loads(str(z["header"]))
        tensors = {}
        for key, m in self.meta.items():
            item = dict(m)
            item["data"] = torch.from_numpy(z[f"data/{key}"].copy())
            item["scales"] = None
            item["scales_data"] = (torch.from_numpy(z[f"scales_data/{key}"].copy())
                                   if f"scales_data/{key}" in z.files else None)
            tensors[key] = item
        self.state = dict(header)
        self.state["tensors"] = tensors

    def decoded(self, key):
        m = self.meta[key]
        dt = torch.float32 if m["pack_kind"] in ("int8_symmetric", "int8_rowwise") else DTYPES[m["packed_dtype"]]
        return from_np(self.z[f"decoded/{key}"], dt)

    def applied(self, name, dtype, key):
        return from_np(self.z[f"applied/{name}/{str(dtype)[6:]}/{key}"], dtype)

    def applied_keys(self):
        return sorted({f.split("/", 3)[3] for f in self.z.files if f.startswith("applied/")})
