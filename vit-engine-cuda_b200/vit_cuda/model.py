"""ViT-B/16 inference module with the reference's surface
(vit_cuda/model.py:18-166 of the reference project): ``ViTCUDA(num_classes,
state_dict, pretrained)`` registers timm-named buffers, ``forward`` returns
logits, ``capture_graph`` records the forward in a CUDA graph and later calls
replay it.

Behind that surface the forward is one call into libvitb200.so
(``vitb200_vit_forward``), which chains the fused sm_100a kernels on the
current stream: im2col -> patch GEMM (+bias +pos) -> 12 x [LN1 -> QKV GEMM ->
attention -> proj GEMM (+bias +residual) -> LN2 -> fc1 GEMM (+bias +GELU) ->
fc2 GEMM (+bias +residual)] -> LN(CLS rows) -> head GEMM. The linear weights are
split once per device (``prepare``); activations are split by the kernel that
produces them. The four block GEMMs run on FP16 splits (three FP16 tensor-core
products, FP32 accuracy at twice the TF32 rate) wherever the weights bound
their input below the split's range, and on TF32 pairs (TF32x3) otherwise;
``operands="tf32"`` keeps every GEMM on TF32 pairs.

``ViTBlockCUDA.forward`` keeps the reference's op-by-op block (the registered
``torch.ops.vit_cuda`` ops) for callers that drive blocks themselves. Under
``torch.compile`` the fused forward is the registered ``vit_cuda::vit_forward``.
"""
from __future__ import annotations

import ctypes
import math
from typing import Optional

import torch
import torch.nn as nn

from . import _lib, library
from ._lib import BlockParams, VitParams, lib
from .split import F16_SAFE_BOUND, block_input_bounds, f16_weight, f16_weight_ok

_BLOCK_KEYS = [
    ("norm1_gamma", "norm1.weight"), ("norm1_beta", "norm1.bias"),
    ("qkv_weight", "attn.qkv.weight"), ("qkv_bias", "attn.qkv.bias"),
    ("proj_weight", "attn.proj.weight"), ("proj_bias", "attn.proj.bias"),
    ("norm2_gamma", "norm2.weight"), ("norm2_beta", "norm2.bias"),
    ("fc1_weight", "mlp.fc1.weight"), ("fc1_bias", "mlp.fc1.bias"),
    ("fc2_weight", "mlp.fc2.weight"), ("fc2_bias", "mlp.fc2.bias"),
]


class ViTBlockCUDA(nn.Module):
    """One pre-LN encoder block with timm-named buffers (reference model.py:18-60)."""

    def __init__(self, state, idx):
        super().__init__()
        prefix = f"blocks.{idx}."
        for attr, key in _BLOCK_KEYS:
            self.register_buffer(attr, state[prefix + key])

    def forward(self, x, scale, eps):
        residual = x
        x = library.layernorm_forward(x, self.norm1_gamma, self.norm1_beta, eps)
        q, k, v = library.qkv_proj(x, self.qkv_weight, self.qkv_bias)
        attn_out = library.flash_attn_2(q, k, v, scale)
        attn_out = library.gemm_bias(attn_out, self.proj_weight, self.proj_bias)
        x = residual + attn_out
        residual = x
        x = library.layernorm_forward(x, self.norm2_gamma, self.norm2_beta, eps)
        mlp_out = library.mlp_forward(x, self.fc1_weight, self.fc1_bias, self.fc2_weight,
                                 self.fc2_bias)[0]
        return residual + mlp_out


def _split_pair(w: torch.Tensor) -> torch.Tensor:
    """TF32 pair [2][N][K] of a 2-D fp32 CUDA weight (K % 4 == 0)."""
    w2 = w.reshape(w.shape[0], -1).contiguous()
    n, k = w2.shape
    if k % 4:
        raise RuntimeError("weight inner dim must be a multiple of 4")
    pair = torch.empty((2, n, k), dtype=torch.float32, device=w2.device)
    _lib.check(lib.vitb200_split_tf32(w2.data_ptr(), n, k, k, pair.data_ptr(), k,
                                      torch.cuda.current_stream().cuda_stream),
               "vitb200_split_tf32")
    return pair


class ViTCUDA(nn.Module):
    def __init__(self, num_classes=1000, state_dict=None, pretrained=True, operands="auto",
                 ln_fold=True):
        super().__init__()
        if operands not in ("auto", "tf32"):
            raise ValueError("operands must be 'auto' or 'tf32'")
        self.operands = operands
        # Fold the LayerNorms before qkv and fc1 into those GEMMs when every
        # block GEMM runs on FP16 splits (vitb200_vit_params.ln_fold): the
        # residual stream's magnitudes must then stay below 32768.
        self.ln_fold = bool(ln_fold)
        if state_dict is None:
            try:
                import timm  # noqa: F401  (reference model.py:67-69)
            except ImportError as e:  # pragma: no cover - timm is not in this image
                raise RuntimeError(
                    "ViTCUDA: pass state_dict= (timm, needed to fetch weights, is not "
                    "installed); vit_cuda.weights.synthetic_state_dict() builds one") from e
            state = timm.create_model("vit_base_patch16_224", pretrained=pretrained).state_dict()
        else:
            state = state_dict

        self.num_classes = num_classes
        self.scale = 1.0 / math.sqrt(64)
        self.eps = 1e-6

        self.register_buffer("patch_weight", state["patch_embed.proj.weight"])
        self.register_buffer("patch_bias", state["patch_embed.proj.bias"])
        cls = state["cls_token"]
        self.register_buffer("cls_token", cls.reshape(1, -1) if cls.dim() != 2 else cls)
        pos = state["pos_embed"]
        self.register_buffer("pos_embed", pos.squeeze(0) if pos.dim() == 3 else pos)
        depth = 0
        while f"blocks.{depth}.norm1.weight" in state:
            depth += 1
        self.blocks = nn.ModuleList([ViTBlockCUDA(state, i) for i in range(depth)])
        self.register_buffer("norm_gamma", state["norm.weight"])
        self.register_buffer("norm_beta", state["norm.bias"])
        self.register_buffer("head_weight", state["head.weight"])
        self.register_buffer("head_bias", state["head.bias"])

        T = self.pos_embed.shape[0]
        grid = int(round(math.sqrt(T - 1)))
        if grid * grid != T - 1:
            raise RuntimeError("pos_embed length must be a square number of patches + 1")
        self.img_size = (grid * 16, grid * 16)
        self.in_chans = self.patch_weight.shape[1] if self.patch_weight.dim() == 4 else 3
        self._prepared = None  # (key, splits, params, blocks_array, keep-alive, split metadata)
        self._imported = None  # split weights given to import_splits
        self._op_id = library.register_model(self)  # torch.ops.vit_cuda.vit_forward
        self._graph = None

    # ----------------------------------------------------------- weights
    def _source_key(self):
        ptrs = tuple(b.data_ptr() for b in self.buffers())
        return (self.patch_weight.device, ptrs)

    def _compute_splits(self) -> tuple[dict, dict]:
        """The split weights on the model's device: tensors named
        ``patch.f16`` (FP16 planes) or ``patch.pair``, ``head.pair`` and per
        block ``blocks.{i}.{gemm}.pair`` (TF32 pair) or ``blocks.{i}.{gemm}.f16``
        (FP16 planes), plus string metadata: ``patch`` and ``blocks.{i}.{gemm}``
        = "f16" | "tf32", the FP16 GEMMs' ``.acc_scale`` and ``blocks.{i}.attn``
        = "f16" | "tf32". The patch GEMM's input is the image itself, whose
        pixels the FP16 path requires below 32768 in magnitude (the im2col
        kernel reports larger ones through the device error)."""
        tensors = {"head.pair": _split_pair(self.head_weight)}
        meta = {}
        pw = self.patch_weight.reshape(self.patch_weight.shape[0], -1).contiguous()
        if self.operands == "auto" and f16_weight_ok(pw):
            tensors["patch.f16"], acc_scale = f16_weight(pw)
            meta["patch"], meta["patch.acc_scale"] = "f16", repr(acc_scale)
        else:
            tensors["patch.pair"] = _split_pair(self.patch_weight)
            meta["patch"] = "tf32"
        for i, blk in enumerate(self.blocks):
            bounds = block_input_bounds(blk, 768)
            for name in ("qkv", "proj", "fc1", "fc2"):
                weight = getattr(blk, f"{name}_weight")
                key = f"blocks.{i}.{name}"
                if (self.operands == "auto" and bounds[name] < F16_SAFE_BOUND
                        and f16_weight_ok(weight)):
                    tensors[key + ".f16"], acc_scale = f16_weight(weight.contiguous())
                    meta[key], meta[key + ".acc_scale"] = "f16", repr(acc_scale)
                else:
                    tensors[key + ".pair"] = _split_pair(weight)
                    meta[key] = "tf32"
            # The FP16 attention: q, k and v within the split's range.
            attn_f16 = (self.operands == "auto" and bounds["q"] < F16_SAFE_BOUND
                        and bounds["k"] < F16_SAFE_BOUND and bounds["v"] < F16_SAFE_BOUND)
            meta[f"blocks.{i}.attn"] = "f16" if attn_f16 else "tf32"
        fold = self.ln_fold and self.operands == "auto" and all(
            meta[f"blocks.{i}.{n}"] == "f16" for i in range(len(self.blocks))
            for n in ("qkv", "proj", "fc1", "fc2"))
        folded = {}
        for i, blk in enumerate(self.blocks if fold else []):
            for name, gamma, beta in (("qkv", blk.norm1_gamma, blk.norm1_beta),
                                      ("fc1", blk.norm2_gamma, blk.norm2_beta)):
                wt = getattr(blk, f"{name}_weight")
                b = getattr(blk, f"{name}_bias")
                wg = (wt * gamma.reshape(1, -1)).contiguous()
                if not f16_weight_ok(wg):
                    fold = False
                    break
                key = f"blocks.{i}.ln_{name}"
                folded[key + ".f16"], acc_scale = f16_weight(wg)
                folded[key + ".c"] = (wt.double() @ gamma.double()).float().contiguous()
                folded[key + ".d"] = (wt.double() @ beta.double() + b.double()).float().contiguous()
                meta[key + ".acc_scale"] = repr(acc_scale)
            if not fold:
                break
        if fold:
            tensors.update(folded)
        meta["ln_fold"] = "1" if fold else "0"
        return tensors, meta

    def export_splits(self) -> tuple[dict, dict]:
        """The split weights prepare() made (for vit_cuda.checkpoint.save_splits)."""
        prepared = self.prepare()
        return dict(prepared[1]), dict(prepared[5])

    def import_splits(self, tensors: dict, meta: dict) -> None:
        """Uses previously exported split weights instead of splitting again
        (vit_cuda.checkpoint.load_splits checks that they match the weights)."""
        dev = self.patch_weight.device
        self._imported = ({k: v.to(dev) for k, v in tensors.items()}, dict(meta))
        self.prepare(force=True)

    def prepare(self, force: bool = False):
        """Splits the linear weights on their device (FP16 splits where the
        block's input bounds allow, TF32 pairs otherwise; ``gemm_operands``
        records the choice per block), or takes split weights given to
        ``import_splits``, and builds the C parameter block. Runs once per
        device / weight storage; call it again with force=True after modifying
        weights in place."""
        key = self._source_key()
        if not force and self._prepared is not None and self._prepared[0] == key:
            return self._prepared
        if not self.patch_weight.is_cuda:
            raise RuntimeError("ViTCUDA: move the model to a CUDA device first (.to('cuda'))")
        for name, buf in self.named_buffers():
            if buf.dtype != torch.float32:
                raise RuntimeError(f"ViTCUDA: buffer {name} must be float32")
        with torch.cuda.device(self.patch_weight.device):
            _lib.check(lib.vitb200_init(), "vitb200_init")
            imported = getattr(self, "_imported", None)
            if imported is not None and imported[0]["head.pair"].device == self.patch_weight.device:
                splits, meta = imported
            else:
                splits, meta = self._compute_splits()
            blocks = (BlockParams * len(self.blocks))()
            keep = []
            self.gemm_operands = []
            ptr = lambda t: t.data_ptr() if t is not None else None  # noqa: E731
            for i, blk in enumerate(self.blocks):
                w = {}
                kinds = {}
                for name in ("qkv", "proj", "fc1", "fc2"):
                    key_ = f"blocks.{i}.{name}"
                    kinds[name] = meta[key_]
                    if meta[key_] == "f16":
                        w[name] = (None, splits[key_ + ".f16"], float(meta[key_ + ".acc_scale"]))
                    else:
                        w[name] = (splits[key_ + ".pair"], None, 0.0)
                attn_f16 = meta[f"blocks.{i}.attn"] == "f16"
                kinds["attn"] = meta[f"blocks.{i}.attn"]
                self.gemm_operands.append(kinds)
                vecs = [blk.norm1_gamma, blk.norm1_beta, blk.qkv_bias, blk.proj_bias,
                        blk.norm2_gamma, blk.norm2_beta, blk.fc1_bias, blk.fc2_bias]
                vecs = [v.contiguous() for v in vecs]
                keep += vecs
                ln = {}
                for name in ("qkv", "fc1"):
                    key_ = f"blocks.{i}.ln_{name}"
                    if meta.get("ln_fold") == "1":
                        ln[name] = (splits[key_ + ".f16"], float(meta[key_ + ".acc_scale"]),
                                    splits[key_ + ".c"], splits[key_ + ".d"])
                    else:
                        ln[name] = (None, 0.0, None, None)
                blocks[i] = BlockParams(
                    vecs[0].data_ptr(), vecs[1].data_ptr(), ptr(w["qkv"][0]), vecs[2].data_ptr(),
                    ptr(w["proj"][0]), vecs[3].data_ptr(), vecs[4].data_ptr(), vecs[5].data_ptr(),
                    ptr(w["fc1"][0]), vecs[6].data_ptr(), ptr(w["fc2"][0]), vecs[7].data_ptr(),
                    ptr(w["qkv"][1]), w["qkv"][2], ptr(w["proj"][1]), w["proj"][2],
                    ptr(w["fc1"][1]), w["fc1"][2], ptr(w["fc2"][1]), w["fc2"][2],
                    1 if attn_f16 else 0, 1.0, 1.0, 1.0,
                    ptr(ln["qkv"][0]), ln["qkv"][1], ptr(ln["qkv"][2]), ptr(ln["qkv"][3]),
                    ptr(ln["fc1"][0]), ln["fc1"][1], ptr(ln["fc1"][2]), ptr(ln["fc1"][3]))
            vecs = {n: getattr(self, n).contiguous() for n in
                    ("patch_bias", "cls_token", "pos_embed", "norm_gamma", "norm_beta",
                     "head_bias")}
            keep += list(vecs.values())
            params = VitParams(
                depth=len(self.blocks), embed_dim=768, num_heads=12,
                mlp_dim=self.blocks[0].fc1_weight.shape[0], patch=16, in_chans=self.in_chans,
                img_h=self.img_size[0], img_w=self.img_size[1], num_classes=self.num_classes,
                ln_eps=self.eps, attn_scale=self.scale,
                patch_w_pair=ptr(splits.get("patch.pair")),
                patch_b=vecs["patch_bias"].data_ptr(),
                cls_token=vecs["cls_token"].data_ptr(), pos_embed=vecs["pos_embed"].data_ptr(),
                blocks=ctypes.cast(blocks, ctypes.POINTER(BlockParams)),
                norm_w=vecs["norm_gamma"].data_ptr(), norm_b=vecs["norm_beta"].data_ptr(),
                head_w_pair=splits["head.pair"].data_ptr(), head_b=vecs["head_bias"].data_ptr(),
                patch_w_f16=ptr(splits.get("patch.f16")),
                patch_acc_scale=(float(meta["patch.acc_scale"])
                                 if meta.get("patch", "tf32") == "f16" else 0.0),
                ln_fold=1 if meta.get("ln_fold") == "1" else 0)
            self.patch_operands = meta.get("patch", "tf32")
            if self.head_weight.shape[0] != self.num_classes:
                raise RuntimeError("head weight rows must equal num_classes")
        self._prepared = (key, splits, params, blocks, keep, meta)
        return self._prepared

    @property
    def params(self) -> VitParams:
        return self.prepare()[2]

    @property
    def ln_folded(self) -> bool:
        """Whether launches below 1024 token rows fold the LayerNorms before
        qkv and fc1 into those GEMMs (vitb200_vit_params.ln_fold)."""
        return self.prepare()[5].get("ln_fold") == "1"

    def workspace_bytes(self, batch: int) -> int:
        return int(lib.vitb200_vit_workspace_bytes(ctypes.byref(self.params), int(batch)))

    def _check_input(self, x: torch.Tensor) -> torch.Tensor:
        if not isinstance(x, torch.Tensor) or not x.is_cuda:
            raise RuntimeError("ViTCUDA: input must be a CUDA tensor")
        if x.dtype != torch.float32:
            raise RuntimeError("ViTCUDA: input must be float32")
        if x.dim() != 4 or x.shape[1] != self.in_chans or tuple(x.shape[2:]) != self.img_size:
            raise RuntimeError(
                f"ViTCUDA: input must be [B, {self.in_chans}, {self.img_size[0]}, "
                f"{self.img_size[1]}], got {list(x.shape)}")
        if x.device != self.patch_weight.device:
            raise RuntimeError("ViTCUDA: input and model must be on the same device")
        return x.contiguous()

    # ----------------------------------------------------------- forward
    def forward(self, x):
        # Under torch.compile the fused forward is one registered custom op.
        if torch.compiler.is_compiling():
            return torch.ops.vit_cuda.vit_forward(x, self._op_id, self.num_classes)
        # CUDA graph replay path (fixed input shape/address), reference model.py:93-99.
        if self._graph is not None:
            self._static_input.copy_(x)
            self._graph.replay()
            return self._static_output
        return self._forward_impl(x)

    def _run(self, fn_name: str, x: torch.Tensor, out_cols: int) -> torch.Tensor:
        x = self._check_input(x)
        params = self.params
        B = x.shape[0]
        out = torch.empty((B, out_cols), dtype=torch.float32, device=x.device)
        nbytes = lib.vitb200_vit_workspace_bytes(ctypes.byref(params), B)
        ws = torch.empty(max(int(nbytes), 1), dtype=torch.uint8, device=x.device)
        fn = getattr(lib, fn_name)
        _lib.check(fn(ctypes.byref(params), x.data_ptr(), out.data_ptr(), B, ws.data_ptr(),
                      ws.numel(), torch.cuda.current_stream().cuda_stream), fn_name)
        return out

    def _forward_impl(self, x):
        return self._run("vitb200_vit_forward", x, self.num_classes)

    def forward_features(self, x):
        """CLS-token features after the final LayerNorm, [B, 768] (the features
        the reference's evaluation scripts use)."""
        return self._run("vitb200_vit_forward_features", x, 768)

    # ------------------------------------------------- layerwise pieces
    def embed(self, x: torch.Tensor) -> torch.Tensor:
        """Token embeddings [B, T, 768] (patch embed + CLS + pos)."""
        x = self._check_input(x)
        params = self.params
        B = x.shape[0]
        T = self.pos_embed.shape[0]
        out = torch.empty((B, T, 768), dtype=torch.float32, device=x.device)
        ws = self._ws(B, x.device)
        _lib.check(lib.vitb200_vit_embed(ctypes.byref(params), x.data_ptr(), out.data_ptr(), B,
                                         ws.data_ptr(), ws.numel(),
                                         torch.cuda.current_stream().cuda_stream),
                   "vitb200_vit_embed")
        return out

    def block(self, layer: int, tokens: torch.Tensor) -> torch.Tensor:
        """Runs encoder block `layer` of the fused path on a copy of tokens [B, T, 768]."""
        params = self.params
        y = tokens.detach().to(torch.float32).contiguous().clone()
        B = y.shape[0]
        ws = self._ws(B, y.device)
        _lib.check(lib.vitb200_vit_block(ctypes.byref(params), int(layer), y.data_ptr(), B,
                                         ws.data_ptr(), ws.numel(),
                                         torch.cuda.current_stream().cuda_stream),
                   "vitb200_vit_block")
        return y

    def head(self, tokens: torch.Tensor):
        """(logits [B, C], features [B, 768]) from final tokens [B, T, 768]."""
        params = self.params
        t = tokens.contiguous()
        B = t.shape[0]
        logits = torch.empty((B, self.num_classes), dtype=torch.float32, device=t.device)
        feats = torch.empty((B, 768), dtype=torch.float32, device=t.device)
        ws = self._ws(B, t.device)
        _lib.check(lib.vitb200_vit_head(ctypes.byref(params), t.data_ptr(), logits.data_ptr(),
                                        feats.data_ptr(), B, ws.data_ptr(), ws.numel(),
                                        torch.cuda.current_stream().cuda_stream),
                   "vitb200_vit_head")
        return logits, feats

    def _ws(self, batch: int, device) -> torch.Tensor:
        nbytes = lib.vitb200_vit_workspace_bytes(ctypes.byref(self.params), batch)
        return torch.empty(max(int(nbytes), 1), dtype=torch.uint8, device=device)

    # ----------------------------------------------------------- graphs
    def capture_graph(self, static_input, num_warmup=3):
        """Capture the full forward pass as a CUDA graph (reference model.py:128-166).

        `static_input` is a CUDA float32 tensor of the exact shape the graph will
        replay; its storage is the graph's input buffer. After capture, `model(x)`
        copies `x` into it and replays the graph."""
        if not static_input.is_cuda:
            raise RuntimeError("capture_graph: static_input must be a CUDA tensor")
        if static_input.dtype != torch.float32:
            raise RuntimeError("capture_graph: static_input must be float32")
        if self._graph is not None:
            raise RuntimeError("capture_graph: a graph is already captured")
        static_input = static_input.contiguous()
        self.eval()
        self.prepare()
        s = torch.cuda.Stream()
        s.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(s):
            with torch.no_grad():
                for _ in range(num_warmup):
                    self._forward_impl(static_input)
        torch.cuda.current_stream().wait_stream(s)
        torch.cuda.synchronize()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            with torch.no_grad():
                self._static_output = self._forward_impl(static_input)
        self._static_input = static_input
        self._graph = graph
        torch.cuda.synchronize()
        return graph

    def release_graph(self):
        """Drops a captured graph; `forward` runs eagerly again."""
        self._graph = None
        self._static_input = None
        self._static_output = None
