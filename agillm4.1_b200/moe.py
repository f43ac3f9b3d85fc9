"""Drop-in MoE block for AGILLM4.1 whose forward runs on the sm_100a kernels.

``MoEFFN`` keeps the reference class's interface (agillm41.py:4323-4460):

* constructor ``MoEFFN(d, mlp_mult=4, experts=4, top_k=1, shared_experts=0,
  shared_mlp_mult=0)`` and the same submodules, so the same state-dict keys:
  ``router.weight``, ``experts.{e}.{0,2}.{weight,bias}``,
  ``shared.{s}.{0,2}.{weight,bias}`` (4324-4351);
* attributes ``d, mlp_mult, num_experts, top_k, num_shared,
  last_router_input, expert_stream, expert_stream_empty_cache,
  expert_stream_stats`` and ``set_expert_stream`` (4353-4365);
* the legacy dense-FFN state-dict seeding of ``_load_from_state_dict``
  (4433-4460);
* ``forward(x[..., d]) -> Tensor[same shape, same dtype]``: the FFN output
  only (the caller adds the residual, agillm41.py:4542, 4547).

The forward calls the fused C-ABI entry point ``agm_moe_forward`` (router ->
dispatch plan -> permute -> grouped FC1/FC2 -> combine) on the current CUDA
stream with no host synchronisation. It refuses CPU tensors (there is no CPU
fallback). With ``set_expert_stream(True)`` the routed experts stay on the host
and only the active ones are copied in for each call.

Training: when autograd needs gradients, the forward runs
``agm_moe_forward_train`` inside an autograd node whose backward is
``agm_moe_backward`` (router, gates, expert FFNs and combine on the B200
kernels), in the two precision modes the reference trains in: one dtype
throughout, or torch.autocast (bf16/fp16) over fp32 master weights with an
fp32 input, as ``Block`` feeds it from its LayerNorm (agillm41.py:4539-4547)
under the reference's ``amp()`` (agillm41.py:3054-3066), shared experts
included.

``install(agillm41)`` rebinds the reference module's ``MoEFFN`` to a subclass
of the reference class that uses this forward, so ``Block`` (4533-4537), the
AR/SAT/NAT inference paths and the pipeline-stage runtime construct it, and
``isinstance(m, agillm41.MoEFFN)`` checks (4475, 7657, 7674, 7685, 7694) hold.
"""
from __future__ import annotations

from typing import Optional

import torch
import torch.nn as nn

from . import ops
from ._lib import MoEKernelError


def _autocast_dtype(device: torch.device) -> Optional[torch.dtype]:
    """The 16-bit dtype torch.autocast runs CUDA ops in here, or None."""
    if device.type != "cuda" or not torch.is_autocast_enabled(device.type):
        return None
    dt = torch.get_autocast_dtype(device.type)
    return dt if dt in (torch.bfloat16, torch.float16) else None


class _MoETrainNode(torch.autograd.Function):
    """Autograd node of the MoE block: ``agm_moe_forward_train`` forward,
    ``agm_moe_backward`` backward. Replaces the graph autograd records through
    agillm41.py:4398-4428 (router Linear, top-k/softmax or top-1
    straight-through gates, index_select, expert Linear/ReLU/Linear, the gate
    product and index_add_).

    Inputs: x [N, d], the residual added last (or None), the router weight, a
    state dict (compute-dtype weights,
    top_k, error checking) and the parameters in the order
    experts.{e}.0.weight, .0.bias, .2.weight, .2.bias for e = 0..E-1, then
    shared.{s}.0.weight, ... for the shared experts; their gradients come
    back as views of the packed [E, ...] / [S, ...] gradient tensors.
    Everything the backward reads is saved with save_for_backward, so
    activation checkpointing (agillm41.py:1202, 4662) can drop and recompute it.

    An expert that received no row is never called by the reference, so its
    parameters get no gradient at all (None), which optimisers treat
    differently from a zero gradient (no weight decay, no moment update). With
    state["empty_grad"] == "none" (the default) the backward reads the
    per-expert row counts (one small device-to-host copy) and returns None for
    such experts; "zero" skips the copy and returns zero gradients.
    """

    @staticmethod
    def forward(ctx, x, residual, w_router, state, *params):
        wr_c, w1, b1, w2, b2 = state["weights"]
        sh = state.get("shared")
        out, saved, counts = ops.moe_forward_train(x, wr_c, w1, b1, w2, b2, state["top_k"], shared=sh,
                                                   residual=residual, check_errors=state["check"], want_counts=True)
        if sh is not None:
            ctx.save_for_backward(saved, wr_c, w1, w2, counts, sh[0], sh[2])
        else:
            ctx.save_for_backward(saved, wr_c, w1, w2, counts)
        ctx.top_k = state["top_k"]
        ctx.check = state["check"]
        ctx.none_for_empty = state.get("empty_grad", "none") == "none"
        ctx.n_experts = w1.shape[0]
        return out

    @staticmethod
    def backward(ctx, dout):
        saved, wr_c, w1, w2, counts, *sw = ctx.saved_tensors
        shared = None
        if sw:
            # only the weights' shapes and pointers matter for the biases here
            shared = (sw[0], None, sw[1], None)
        res = ops.moe_backward(dout.contiguous(), saved, wr_c, w1, w2, ctx.top_k, shared=shared,
                               check_errors=ctx.check)
        dx, dwr, dw1, db1, dw2, db2 = res[:6]
        used = counts.cpu().tolist() if ctx.none_for_empty else None
        grads = []
        for e in range(ctx.n_experts):
            if used is not None and used[e] == 0:
                grads += [None, None, None, None]
            else:
                grads += [dw1[e], db1[e], dw2[e], db2[e]]
        if sw:
            dws1, dsb1, dws2, dsb2 = res[6]
            for s in range(dws1.shape[0]):
                grads += [dws1[s], dsb1[s], dws2[s], dsb2[s]]
        # the residual enters the output unchanged: its gradient is dout
        dres = dout if ctx.needs_input_grad[1] else None
        return (dx if ctx.needs_input_grad[0] else None, dres, dwr if ctx.needs_input_grad[2] else None, None, *grads)


class _MoEAuxNode(torch.autograd.Function):
    """Auxiliary router losses of one MoE module (agillm41.py:4477-4491) on the
    B200 kernels: ``agm_moe_aux_forward`` recomputes the router logits from the
    stashed input and reduces the load-balance and router-z terms to one fp32
    scalar; ``agm_moe_aux_backward`` gives the router weight's gradient (the
    stashed input is detached in the reference, so it gets none).

    ``cdt`` is the autocast dtype when the call runs under torch.autocast (the
    router Linear then computes in 16 bits on casts of the fp32 input and
    weight, and the weight's gradient comes back through the cast), else None.
    """

    @staticmethod
    def forward(ctx, w_router, x, aux_coef, z_coef, cdt, check):
        wc, xc = w_router, x
        if cdt is not None and w_router.dtype != cdt:
            wc = ops.cast_f32(w_router, cdt) if w_router.dtype == torch.float32 else w_router.to(cdt)
        if xc.dtype != wc.dtype:
            xc = ops.cast_f32(xc, wc.dtype) if xc.dtype == torch.float32 else xc.to(wc.dtype)
        loss, saved = ops.moe_aux_forward(xc.contiguous(), wc.contiguous(), aux_coef, z_coef, check_errors=check)
        ctx.save_for_backward(saved, xc, wc)
        ctx.w_dtype = w_router.dtype
        return loss

    @staticmethod
    def backward(ctx, gl):
        saved, xc, wc = ctx.saved_tensors
        dw = ops.moe_aux_backward(gl, xc, wc, saved)
        if dw.dtype != ctx.w_dtype:
            dw = dw.to(ctx.w_dtype)  # the autocast cast's backward
        return dw, None, None, None, None, None


def collect_moe_aux(model, aux_coef=0.0, z_coef=0.0):
    """``_collect_moe_aux`` (agillm41.py:4463-4492) with each module's losses
    computed by the fused auxiliary-loss kernels: sum and clear the
    load-balance / router-z losses of every B200 MoE module in ``model``.

    Same contract as the reference: the router is recomputed on the detached
    input each module stashed during its training forward (so it works with
    gradient checkpointing and only ``router.weight`` gets a gradient), every
    stash is cleared, and the result is a scalar fp32 tensor to add to the
    loss before ``backward()``, or 0.0 when both coefficients are <= 0 or
    nothing was stashed. The module losses are added in module order.
    """
    total = None
    for m in model.modules():
        if isinstance(m, _B200Forward):
            inp = m.last_router_input
            m.last_router_input = None
            if inp is None or (aux_coef <= 0 and z_coef <= 0):
                continue
            w = m.router.weight
            router_in = inp.to(w.dtype) if inp.dtype != w.dtype else inp  # agillm41.py:4481
            if router_in.device.type != "cuda":
                raise MoEKernelError("collect_moe_aux: the stashed router input is not a CUDA tensor")
            flat = router_in.reshape(-1, router_in.shape[-1])
            loss = _MoEAuxNode.apply(w, flat, float(aux_coef), float(z_coef), _autocast_dtype(flat.device),
                                     bool(m.check_device_errors))
            total = loss if total is None else total + loss
    return total if total is not None else 0.0


class _B200Forward:
    """Forward of the MoE block on the B200 kernels (mixed into the module classes)."""

    # Set to True to synchronise and check the device error word after each
    # forward (tests do; the hot path does not).
    check_device_errors = False
    # Where the router logits come from:
    #   "kernel"         - the router kernel: fp32 accumulation of the bf16/fp16
    #                      products, one rounding to the activation dtype;
    #   "reference_gemm" - the reference's own call, `router(x).float()`
    #                      (agillm41.py:4398-4399, a library GEMM), then the
    #                      same selection kernel. On the same GPU this gives
    #                      routing bit-identical to the reference, whose
    #                      library GEMM may round its split-K partial sums.
    router_logits = "kernel"
    # Gradient of an expert that received no row in a training forward:
    #   "none" - None, as in the reference, which never calls such an expert
    #            (costs one small device-to-host copy per backward);
    #   "zero" - zero tensors, without that copy.
    empty_expert_grad = "none"

    def _packed_weights(self, device: torch.device, dtype: torch.dtype):
        """Expert weights as contiguous [E, ...] device tensors, with the
        module's parameters re-pointed at views of them so that in-place
        updates (load_state_dict, optimiser steps) keep the pack current."""
        experts = list(self.experts)
        params = [p for ex in experts for p in (ex[0].weight, ex[0].bias, ex[2].weight, ex[2].bias)]
        shared = list(self.shared) if getattr(self, "shared", None) is not None else []
        sparams = [p for ex in shared for p in (ex[0].weight, ex[0].bias, ex[2].weight, ex[2].bias)]
        key = (device, dtype) + tuple(p.data_ptr() for p in params + sparams)
        cache = getattr(self, "_b200_pack", None)
        if cache is not None and cache[0] == key:
            return cache[1]
        for p in params + sparams:
            if p.device != device or p.dtype != dtype:
                raise MoEKernelError(f"expert parameters must be on {device} in {dtype}, found {p.device}/{p.dtype}")

        def stack(mods, i, attr):
            return torch.stack([getattr(m[i], attr).detach() for m in mods]).contiguous()

        with torch.no_grad():
            w1, b1, w2, b2 = stack(experts, 0, "weight"), stack(experts, 0, "bias"), \
                stack(experts, 2, "weight"), stack(experts, 2, "bias")
            for e, ex in enumerate(experts):
                ex[0].weight.data = w1[e]
                ex[0].bias.data = b1[e]
                ex[2].weight.data = w2[e]
                ex[2].bias.data = b2[e]
            sh = None
            if shared:
                sw1, sb1, sw2, sb2 = stack(shared, 0, "weight"), stack(shared, 0, "bias"), \
                    stack(shared, 2, "weight"), stack(shared, 2, "bias")
                for s, ex in enumerate(shared):
                    ex[0].weight.data = sw1[s]
                    ex[0].bias.data = sb1[s]
                    ex[2].weight.data = sw2[s]
                    ex[2].bias.data = sb2[s]
                sh = (sw1, sb1, sw2, sb2)
        packed = (w1, b1, w2, b2, sh)
        key = (device, dtype) + tuple(p.data_ptr() for p in params + sparams)
        self._b200_pack = (key, packed)
        return packed

    def _expert_params(self):
        experts = [p for ex in self.experts for p in (ex[0].weight, ex[0].bias, ex[2].weight, ex[2].bias)]
        shared = list(self.shared) if getattr(self, "shared", None) is not None else []
        return experts + [p for ex in shared for p in (ex[0].weight, ex[0].bias, ex[2].weight, ex[2].bias)]

    def _compute_weights(self, device: torch.device, master_dtype: torch.dtype, compute_dtype: torch.dtype):
        """((router, w1, b1, w2, b2), shared (ws1, sb1, ws2, sb2) or None) in
        the compute dtype. Same dtype: the packed parameters themselves.
        Autocast: their 16-bit casts, made once per change of the parameters
        (the version counters of the parameters key the cache, so an
        optimiser step or load_state_dict recasts)."""
        w1, b1, w2, b2, sh = self._packed_weights(device, master_dtype)
        wr = self.router.weight
        if compute_dtype == master_dtype:
            return (wr.detach().contiguous(), w1, b1, w2, b2), sh
        params = [wr] + self._expert_params()
        key = (device, compute_dtype) + tuple((p.data_ptr(), p._version) for p in params)
        cache = getattr(self, "_b200_cast", None)
        if cache is not None and cache[0] == key:
            return cache[1]
        with torch.no_grad():
            cast = tuple(ops.cast_f32(t.detach(), compute_dtype) for t in (wr, w1, b1, w2, b2))
            csh = None if sh is None else tuple(ops.cast_f32(t, compute_dtype) for t in sh)
        self._b200_cast = (key, (cast, csh))
        return cast, csh

    # ---- expert streaming (agillm41.py:4367-4379, 7656-7668) ----
    def _host_expert_pack(self, dtype: torch.dtype):
        """The routed experts' weights (on the host, as the reference's block
        streaming leaves them) packed into page-locked [E, ...] tensors, made
        again whenever a parameter changes (pointer or version)."""
        experts = list(self.experts)
        params = [p for ex in experts for p in (ex[0].weight, ex[0].bias, ex[2].weight, ex[2].bias)]
        key = (dtype,) + tuple((p.data_ptr(), p._version, p.device) for p in params)
        cache = getattr(self, "_b200_host_pack", None)
        if cache is not None and cache[0] == key:
            return cache[1]
        with torch.no_grad():
            pack = []
            for i, attr in ((0, "weight"), (0, "bias"), (2, "weight"), (2, "bias")):
                t = torch.stack([getattr(ex[i], attr).detach().to("cpu", dtype) for ex in experts])
                pack.append(t.contiguous().pin_memory())
        self._b200_host_pack = (key, tuple(pack))
        return tuple(pack)

    def _forward_expert_stream(self, flat: torch.Tensor) -> torch.Tensor:
        """MoEFFN.forward with the routed experts resident on the host
        (`set_expert_stream(True)`, agillm41.py:4362-4379): route on the GPU,
        read the per-expert row counts, copy only the active experts' weights
        to the GPU (page-locked, on a side stream while the rows are permuted)
        and run the same kernels. Each active expert is copied once, where the
        reference copies it once per (rank, expert) call. The output equals the
        device-resident forward's bit for bit; `expert_stream_stats` counts
        loads and tokens as the reference does (one load per (rank, expert)
        call with rows, its rows as tokens)."""
        if torch.is_grad_enabled() and (flat.requires_grad or any(p.requires_grad for p in self.parameters())):
            raise MoEKernelError("expert_stream (host-resident experts) runs the inference forward only; call it "
                                 "under torch.no_grad()")
        wr = self.router.weight
        if not wr.is_cuda or wr.device != flat.device:
            raise MoEKernelError("expert_stream: the router weight must be on the input's GPU")
        if flat.dtype != wr.dtype:
            raise MoEKernelError(f"input dtype {flat.dtype} differs from the router weight dtype {wr.dtype}")
        dev, dt = flat.device, flat.dtype
        flat = flat.contiguous()
        n, d = flat.shape
        E, k = self.num_experts, self.top_k
        w1h, b1h, w2h, b2h = self._host_expert_pack(dt)
        H = w1h.shape[1]
        with torch.no_grad():
            wrc = wr.detach().contiguous()
            idx, gates, hist, _ = ops.router_topk(flat, wrc, k)
            plan = ops.dispatch_plan(hist, n, k)
            per_rank = torch.stack([torch.bincount(idx[:, r].long(), minlength=E) for r in range(k)])
            per_rank = per_rank.cpu()                    # the one host synchronisation
            active = [e for e in range(E) if int(per_rank[:, e].sum()) > 0]
            st = self.expert_stream_stats
            st["loads"] = int(st.get("loads", 0)) + int((per_rank > 0).sum())
            st["tokens"] = int(st.get("tokens", 0)) + int(per_rank.sum())
            cur = torch.cuda.current_stream(dev)
            side = torch.cuda.Stream(dev)
            side.wait_stream(cur)
            w1 = torch.empty(E, H, d, dtype=dt, device=dev)
            b1 = torch.empty(E, H, dtype=dt, device=dev)
            w2 = torch.empty(E, d, H, dtype=dt, device=dev)
            b2 = torch.empty(E, d, dtype=dt, device=dev)
            with torch.cuda.stream(side):
                for e in active:
                    for dst, src in ((w1, w1h), (b1, b1h), (w2, w2h), (b2, b2h)):
                        dst[e].copy_(src[e], non_blocking=True)
            x_perm, row_of = ops.permute(flat, idx, plan, E)
            cur.wait_stream(side)
            for t in (w1, b1, w2, b2):
                t.record_stream(side)
            max_tiles = plan["tile_expert"].numel()
            h = ops.grouped_gemm(x_perm, w1, b1, relu=True, tile_group=plan["tile_expert"],
                                 num_tiles=plan["num_tiles"], max_tiles=max_tiles)
            y = ops.grouped_gemm(h, w2, b2, relu=False, tile_group=plan["tile_expert"], num_tiles=plan["num_tiles"],
                                 max_tiles=max_tiles)
            shared_y = None
            if getattr(self, "shared", None) is not None:
                outs = [ops.grouped_gemm(ops.grouped_gemm(flat, ex[0].weight.detach().contiguous(),
                                                          ex[0].bias.detach().contiguous(), relu=True),
                                         ex[2].weight.detach().contiguous(), ex[2].bias.detach().contiguous(),
                                         relu=False)
                        for ex in self.shared]
                shared_y = torch.stack(outs)
            out = ops.combine(y, row_of, gates, shared_y)
            del w1, b1, w2, b2, h, y, x_perm
        if self.expert_stream_empty_cache:
            torch.cuda.empty_cache()
        return out

    def forward(self, x: torch.Tensor) -> torch.Tensor:  # agillm41.py:4389-4431
        return self._forward_impl(x, None)

    def forward_residual(self, x: torch.Tensor, residual: torch.Tensor) -> torch.Tensor:
        """``residual + self(x)`` with the add done by the combine kernel: the
        tail of Block.forward (`x + self.ff(self.ln2(x))`, agillm41.py:4547),
        x being the LayerNorm output and residual the block input. Same
        value and gradients as the two separate ops."""
        if residual.shape != x.shape:
            raise MoEKernelError(f"residual shape {tuple(residual.shape)} differs from {tuple(x.shape)}")
        return self._forward_impl(x, residual)

    def forward_block(self, x: torch.Tensor, ln: nn.Module) -> torch.Tensor:
        """``x + self(ln(x))``: the whole FFN half of Block.forward
        (agillm41.py:4547, `x + self.ff(self.ln2(x))`; with a KV cache pass
        x + y, 4543), x being the block input and ``ln`` its ``ln2``. In
        inference (no gradient, device-resident experts, kernel routing, one
        dtype throughout) the LayerNorm runs on this library's HBM-bound kernel
        and the residual is added in the combine (agm_moe_forward_residual);
        otherwise it is ``self.forward_residual(ln(x), x)`` with torch's
        LayerNorm. The LayerNorm's statistics are reduced in another order than
        torch's, so the result is within the bf16 parity tolerance of the
        reference, not bit-identical to it."""
        wr = self.router.weight
        flat = x.reshape(-1, x.shape[-1])
        fusable = (
            isinstance(ln, nn.LayerNorm) and ln.elementwise_affine and tuple(ln.normalized_shape) == (x.shape[-1],)
            and ln.weight is not None and ln.bias is not None
            and not (torch.is_grad_enabled() and (x.requires_grad or any(p.requires_grad for p in self.parameters())
                                                  or ln.weight.requires_grad))
            and not self.training and not self.expert_stream and self.router_logits == "kernel"
            and flat.is_cuda and wr.is_cuda and flat.dtype == wr.dtype == ln.weight.dtype == ln.bias.dtype
            and _autocast_dtype(flat.device) is None
            and x.shape[-1] <= (1536 if flat.dtype == torch.float32 else 2048)
        )
        if not fusable:
            return self.forward_residual(ln(x), x)
        w1, b1, w2, b2, sh = self._packed_weights(flat.device, flat.dtype)
        out = ops.moe_block_forward(flat.contiguous(), ln.weight.detach().contiguous(), ln.bias.detach().contiguous(),
                                    float(ln.eps), wr.detach().contiguous(), w1, b1, w2, b2, self.top_k, shared=sh,
                                    check_errors=self.check_device_errors)
        return out.reshape(x.shape)

    def _forward_impl(self, x: torch.Tensor, residual: Optional[torch.Tensor]) -> torch.Tensor:
        orig_shape = x.shape
        flat = x.reshape(-1, orig_shape[-1])
        res = None if residual is None else residual.reshape(-1, orig_shape[-1])
        if self.training:
            # agillm41.py:4392-4397: stash the detached input for _collect_moe_aux.
            self.last_router_input = flat.detach()
        if not flat.is_cuda:
            raise MoEKernelError("MoEFFN (B200) runs on CUDA tensors only; there is no CPU path")
        if res is not None and (not res.is_cuda or res.device != flat.device):
            raise MoEKernelError("the residual must be on the input's GPU")
        if self.expert_stream:
            out = self._forward_expert_stream(flat)
            return (out if res is None else res + out).reshape(orig_shape)
        wr = self.router.weight
        amp = _autocast_dtype(flat.device)
        amp_mode = amp is not None and wr.dtype == torch.float32
        if amp_mode and flat.dtype != torch.float32:
            raise MoEKernelError(f"under autocast the MoE input must be fp32 (the LayerNorm output), not {flat.dtype}")
        if not amp_mode and flat.dtype != wr.dtype:
            raise MoEKernelError(f"input dtype {flat.dtype} differs from the weight dtype {wr.dtype}")
        params = self._expert_params()
        grad = torch.is_grad_enabled() and (flat.requires_grad or wr.requires_grad
                                            or any(p.requires_grad for p in params))
        if grad or amp_mode:
            if self.router_logits != "kernel":
                raise MoEKernelError("training and autocast route with the router kernel's logits only")
            weights, shared = self._compute_weights(flat.device, wr.dtype, amp if amp_mode else wr.dtype)
            flat = flat.contiguous()
            if res is not None and res.dtype != flat.dtype:
                raise MoEKernelError(f"residual dtype {res.dtype} differs from the input dtype {flat.dtype}")
            if grad or (res is not None and res.requires_grad and torch.is_grad_enabled()):
                state = {"weights": weights, "shared": shared, "top_k": self.top_k,
                         "check": self.check_device_errors, "empty_grad": self.empty_expert_grad}
                out = _MoETrainNode.apply(flat, None if res is None else res.contiguous(), wr, state, *params)
            else:
                out, _ = ops.moe_forward_train(flat, *weights, self.top_k, shared=shared,
                                               residual=None if res is None else res.contiguous(),
                                               check_errors=self.check_device_errors)
            return out.reshape(orig_shape)
        w1, b1, w2, b2, sh = self._packed_weights(flat.device, flat.dtype)
        flat = flat.contiguous()
        logits_in = None
        if self.router_logits == "reference_gemm":
            logits_in = self.router(flat).float()
        elif self.router_logits != "kernel":
            raise MoEKernelError(f"router_logits must be 'kernel' or 'reference_gemm', not {self.router_logits!r}")
        if res is not None and res.dtype != flat.dtype:
            raise MoEKernelError(f"residual dtype {res.dtype} differs from the input dtype {flat.dtype}")
        if res is not None and logits_in is None:
            out = ops.moe_forward_residual(flat, res.contiguous(), wr.detach().contiguous(), w1, b1, w2, b2,
                                           self.top_k, shared=sh, check_errors=self.check_device_errors)
            return out.reshape(orig_shape)
        out = ops.moe_forward(flat, wr.detach().contiguous(), w1, b1, w2, b2, self.top_k, shared=sh,
                              check_errors=self.check_device_errors, logits_in=logits_in)
        if res is not None:
            out = res + out
        return out.reshape(orig_shape)


    def forward_host(self, x_host: torch.Tensor, out_host: Optional[torch.Tensor] = None,
                     chunk_tokens: int = ops.DEFAULT_CHUNK_TOKENS) -> torch.Tensor:
        """The forward for activations in host memory: x_host [..., d] on the CPU
        (page-locked for overlap) -> output on the CPU, same shape and dtype.
        Copies and compute overlap chunk by chunk on the module's GPU; the
        result is ready when this returns (it synchronises the stream)."""
        orig_shape = x_host.shape
        flat = x_host.reshape(-1, orig_shape[-1])
        if flat.is_cuda:
            return self.forward(x_host)
        if torch.is_grad_enabled() and any(p.requires_grad for p in self.parameters()):
            raise MoEKernelError("MoEFFN (B200) implements the inference forward only; run it under torch.no_grad()")
        wr = self.router.weight
        if not wr.is_cuda:
            raise MoEKernelError("MoEFFN (B200): move the module to a CUDA device first")
        if flat.dtype != wr.dtype:
            raise MoEKernelError(f"input dtype {flat.dtype} differs from the weight dtype {wr.dtype}")
        w1, b1, w2, b2, sh = self._packed_weights(wr.device, wr.dtype)
        out = None if out_host is None else out_host.reshape(-1, orig_shape[-1])
        out = ops.moe_forward_host(flat.contiguous(), wr.detach().contiguous(), w1, b1, w2, b2, self.top_k,
                                   shared=sh, out_host=out, chunk_tokens=chunk_tokens,
                                   check_errors=self.check_device_errors)
        torch.cuda.current_stream(wr.device).synchronize()
        return out.reshape(orig_shape)


class MoEFFN(_B200Forward, nn.Module):
    """AGILLM4.1 MoE feed-forward block (reference interface, B200 forward)."""

    def __init__(self, d: int, mlp_mult: int = 4, experts: int = 4, top_k: int = 1,
                 shared_experts: int = 0, shared_mlp_mult: int = 0):
        super().__init__()
        # agillm41.py:4324-4360
        self.d = int(d)
        self.mlp_mult = max(1, int(mlp_mult))
        self.num_experts = max(1, int(experts))
        self.top_k = min(max(1, int(top_k)), self.num_experts)
        hidden = self.mlp_mult * self.d
        self.router = nn.Linear(self.d, self.num_experts, bias=False)
        self.experts = nn.ModuleList([
            nn.Sequential(nn.Linear(self.d, hidden), nn.ReLU(), nn.Linear(hidden, self.d))
            for _ in range(self.num_experts)
        ])
        self.num_shared = max(0, int(shared_experts))
        if self.num_shared > 0:
            shidden = max(1, int(shared_mlp_mult) or self.mlp_mult) * self.d
            self.shared = nn.ModuleList([
                nn.Sequential(nn.Linear(self.d, shidden), nn.ReLU(), nn.Linear(shidden, self.d))
                for _ in range(self.num_shared)
            ])
            for blk in self.shared:  # zero-initialised output layer: a no-op at step 0
                nn.init.zeros_(blk[2].weight)
                nn.init.zeros_(blk[2].bias)
        else:
            self.shared = None
        self.last_router_input = None
        self.expert_stream = False
        self.expert_stream_empty_cache = True
        self.expert_stream_stats = {"loads": 0, "tokens": 0}

    def set_expert_stream(self, enabled: bool, empty_cache: bool = True):  # agillm41.py:4362-4365
        self.expert_stream = bool(enabled)
        self.expert_stream_empty_cache = bool(empty_cache)
        return self

    def _load_from_state_dict(self, state_dict, prefix, local_metadata, strict, missing_keys, unexpected_keys,
                              error_msgs):
        # agillm41.py:4433-4460: a dense FFN checkpoint (`ff.0.*`, `ff.2.*`)
        # seeds every expert with the same weights; the router keeps its init.
        legacy = ("0.weight", "0.bias", "2.weight", "2.bias")
        seeded = False
        for e, expert in enumerate(self.experts):
            expert_state = expert.state_dict()
            for suffix in legacy:
                src = state_dict.get(prefix + suffix)
                dst_key = prefix + f"experts.{e}." + suffix
                tgt = expert_state.get(suffix)
                if dst_key not in state_dict and torch.is_tensor(src) and torch.is_tensor(tgt) \
                        and tuple(src.shape) == tuple(tgt.shape):
                    state_dict[dst_key] = src
                    seeded = True
        if seeded and prefix + "router.weight" not in state_dict:
            state_dict[prefix + "router.weight"] = self.router.weight.detach().clone()
        if seeded:
            for suffix in legacy:
                state_dict.pop(prefix + suffix, None)
        return super()._load_from_state_dict(state_dict, prefix, local_metadata, strict, missing_keys,
                                             unexpected_keys, error_msgs)


def _fused_block_forward(self, x, mask, kv=None, use_cache=False, total_seq_len=None):
    """Block.forward (agillm41.py:4539-4547) with the MoE FFN's residual add
    done by its combine kernel (`x + ff(ln2(x))` as one call) and, when the
    Block was installed with ``fuse_layernorm``, ln2 on this library's
    LayerNorm kernel in inference; any other ff runs the reference's own
    forward."""
    ff = self.ff
    if not isinstance(ff, _B200Forward):
        return self._reference_block_forward(x, mask, kv=kv, use_cache=use_cache, total_seq_len=total_seq_len)

    def ffn_half(r):
        if getattr(self, "_fuse_layernorm", False):
            return ff.forward_block(r, self.ln2)
        return ff.forward_residual(self.ln2(r), r)

    if use_cache:
        y, new_kv = self.mha(self.ln1(x), mask, rel_bias_tokens=total_seq_len, kv_cache=kv, use_cache=True)
        return ffn_half(x + y), new_kv  # the reference's `x + y + ff(ln2(x + y))`
    n = x.size(1)
    x = x + self.mha(self.ln1(x), mask, rel_bias_tokens=n)
    return ffn_half(x)


def install(agillm41_module, name: str = "MoEFFN", fuse_residual: bool = False, fuse_aux: bool = True,
            fuse_layernorm: bool = False):
    """Rebind ``agillm41_module.MoEFFN`` to a subclass of the reference class
    whose forward runs on the B200 kernels. Returns the new class.

    Everything except ``forward`` (constructor, state-dict shim, expert
    streaming toggles, aux-loss stash) is inherited from the reference class.
    Modules built after the call (``Block``, ``Encoder``, the inference and
    pipeline-stage runtimes) use it.

    ``fuse_residual``: also rebind ``Block`` to a subclass whose forward adds
    the residual inside the MoE block's combine kernel (same values and
    gradients, one elementwise pass less per layer).

    ``fuse_layernorm`` (implies ``fuse_residual``): that Block's inference
    forward also runs ln2 on this library's LayerNorm kernel
    (:meth:`forward_block`); training keeps torch's LayerNorm.

    ``fuse_aux``: also rebind ``_collect_moe_aux`` (called by the training
    steps, agillm41.py:1378, 6798) to :func:`collect_moe_aux`, which computes
    the auxiliary router losses of the B200 modules with the fused kernels.
    """
    ref_cls = getattr(agillm41_module, name)
    if getattr(ref_cls, "_is_b200", False):
        cls = ref_cls
    else:
        cls = type(name, (_B200Forward, ref_cls), {"_is_b200": True, "_reference_class": ref_cls,
                                                   "__module__": ref_cls.__module__})
        setattr(agillm41_module, name, cls)
    block = getattr(agillm41_module, "Block", None)
    if (fuse_residual or fuse_layernorm) and block is not None and not getattr(block, "_is_b200", False):
        fused = type("Block", (block,), {"_is_b200": True, "_reference_class": block,
                                         "_reference_block_forward": block.forward,
                                         "_fuse_layernorm": bool(fuse_layernorm),
                                         "forward": _fused_block_forward, "__module__": block.__module__})
        setattr(agillm41_module, "Block", fused)
    aux = getattr(agillm41_module, "_collect_moe_aux", None)
    if fuse_aux and aux is not None and not getattr(aux, "_is_b200", False):
        def _collect(model, aux_coef=0.0, z_coef=0.0):
            return collect_moe_aux(model, aux_coef, z_coef)
        _collect._is_b200 = True
        _collect._reference_function = aux
        _collect.__doc__ = collect_moe_aux.__doc__
        setattr(agillm41_module, "_collect_moe_aux", _collect)
    return cls


def uninstall(agillm41_module, name: str = "MoEFFN") -> None:
    for attr in (name, "Block"):
        cls = getattr(agillm41_module, attr, None)
        if getattr(cls, "_is_b200", False):
            setattr(agillm41_module, attr, cls._reference_class)
    aux = getattr(agillm41_module, "_collect_moe_aux", None)
    if getattr(aux, "_is_b200", False):
        setattr(agillm41_module, "_collect_moe_aux", aux._reference_function)
