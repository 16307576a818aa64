"""Tensor-parallel decode step of a Llama-architecture decoder whose linear
layers are held packed (one process per GPU).

The reference models this step only as bytes (KrishnaI2424/Dequant_Project
``dequant/byte_model.py:179-251``: quantized projections and LM head, fp16 KV
cache, one row of the embedding); this module runs it, with every linear layer
going through the fused dequant + GEMV of this package:

* per layer: RMSNorm -> QKV (column-parallel, this rank's query and KV heads
  fused into one packed matrix) -> RoPE -> KV-cache append -> attention over
  the cache -> O (row-parallel over the same heads, one all-reduce) ->
  residual -> RMSNorm -> gate/up (column-parallel, fused) -> SwiGLU -> down
  (row-parallel, one all-reduce) -> residual;
* then the final RMSNorm and the LM head (column-parallel over the
  vocabulary, quantized like the layers) whose slices are all-gathered.

Weights are random N(0, 0.02) fp16 drawn per matrix from a seeded generator on
the model's device, quantized with the packer and then sharded with
``tensor_parallel``, so every tensor-parallel width holds exactly the packed
codes, scales and zero-points of the single-GPU model. Norm weights are ones
(Llama's initialisation); the KV cache of the first ``kv_len`` positions is
N(0, 1) fp16.

``PackedModel`` holds the full packed weights of a model (the same values the
seeded construction produces) and saves/loads them in the ``packed_io``
format, so a large model is quantized once and then only loaded.

``DecodeGraph`` captures one step at a fixed position into a CUDA graph (the
collectives included) for timing; eager ``step`` takes any position.
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import Callable

import torch
import torch.nn.functional as F

from dequant_project_b200 import decode_ops as ops
from dequant_project_b200.packer import PackedWeight, QuantConfig, quantize_tensor
from dequant_project_b200.tensor_parallel import (intermediate_bounds, shard_columns,
                                                  shard_rows, split_bounds)


@dataclass(frozen=True)
class DecoderConfig:
    """Architecture of a Llama-style decoder."""

    n_layers: int
    hidden: int
    n_heads: int
    n_kv_heads: int
    intermediate: int
    vocab: int
    rope_theta: float = 10000.0
    eps: float = 1e-5

    @property
    def head_dim(self) -> int:
        return self.hidden // self.n_heads


LLAMA2_7B = DecoderConfig(32, 4096, 32, 32, 11008, 32000)
LLAMA3_70B = DecoderConfig(80, 8192, 64, 8, 28672, 128256, rope_theta=500000.0)


def cat_rows(parts: list[PackedWeight]) -> PackedWeight:
    """Row-wise concatenation of packed weights of one format and K (the rows
    of each part keep their own scales and zero-points)."""
    cfg, k = parts[0].config, parts[0].shape[1]
    if any(p.config != cfg or p.shape[1] != k for p in parts):
        raise ValueError("cat_rows needs parts of one format and one K")
    zeros = None if parts[0].zeros is None else torch.cat([p.zeros for p in parts])
    return PackedWeight(qweight=torch.cat([p.qweight for p in parts]),
                        scales=torch.cat([p.scales for p in parts]), zeros=zeros,
                        config=cfg, shape=(sum(p.shape[0] for p in parts), k))


def rope_tables(head_dim: int, theta: float, positions: int, device) -> tuple:
    """cos/sin [positions, head_dim] (fp32) of the rotate-half RoPE."""
    inv = theta ** (-torch.arange(0, head_dim, 2, dtype=torch.float64, device=device) / head_dim)
    ang = torch.arange(positions, dtype=torch.float64, device=device)[:, None] * inv[None, :]
    ang = torch.cat([ang, ang], dim=-1)
    return ang.cos().float(), ang.sin().float()


def _default_linear(x: torch.Tensor, pw: PackedWeight) -> torch.Tensor:
    from dequant_project_b200 import quant_linear as ql
    if x.shape[0] <= ql.MAX_M:
        return ql.gemv(x, pw)
    return F.linear(x, ql.dequantize_cuda(pw))


LAYER_MATRICES = ("q", "k", "v", "o", "gate", "up", "down")


def layer_shapes(cfg: DecoderConfig) -> dict[str, tuple[int, int]]:
    """[N, K] of each linear layer of one decoder layer (full, unsharded)."""
    d = cfg.head_dim
    return {"q": (cfg.n_heads * d, cfg.hidden), "k": (cfg.n_kv_heads * d, cfg.hidden),
            "v": (cfg.n_kv_heads * d, cfg.hidden), "o": (cfg.hidden, cfg.n_heads * d),
            "gate": (cfg.intermediate, cfg.hidden), "up": (cfg.intermediate, cfg.hidden),
            "down": (cfg.hidden, cfg.intermediate)}


class SeededWeights:
    """Random N(0, 0.02) fp16 weights, one seeded draw per matrix on
    ``device``, quantized on request (the default weight source)."""

    def __init__(self, qcfg: QuantConfig, seed: int, device):
        self.qcfg, self.seed, self.device = qcfg, seed, device
        self.gen = torch.Generator(device=device)

    def _index(self, name: str) -> int:
        if name == "embed":
            return 1
        if name == "lm_head":
            return 2
        _, layer, mat = name.split(".")
        return 16 * (int(layer) + 1) + LAYER_MATRICES.index(mat)

    def tensor(self, name: str, shape) -> torch.Tensor:
        self.gen.manual_seed(self.seed * 1_000_003 + self._index(name))
        w = torch.randn(shape, generator=self.gen, device=self.device, dtype=torch.float32)
        return (w * 0.02).to(torch.float16)

    def packed(self, name: str, shape) -> PackedWeight:
        return quantize_tensor(self.tensor(name, shape), self.qcfg)


class PackedModel:
    """Full (unsharded) packed weights of a decoder held in memory: the
    layers' linears as ``layers.<i>.<q|k|v|o|gate|up|down>``, the LM head as
    ``lm_head`` (packed or fp16) and the fp16 embedding as ``embed``."""

    def __init__(self, cfg: DecoderConfig, qcfg: QuantConfig, packed: dict, tensors: dict):
        self.cfg, self.qcfg, self.packed_weights, self.tensors = cfg, qcfg, packed, tensors

    def packed(self, name: str, shape) -> PackedWeight:
        pw = self.packed_weights[name]
        if tuple(pw.shape) != tuple(shape) or pw.config != self.qcfg:
            raise ValueError(f"{name}: stored {pw.shape} {pw.config}, expected {tuple(shape)} "
                             f"{self.qcfg}")
        return pw

    def tensor(self, name: str, shape) -> torch.Tensor:
        t = self.tensors[name]
        if tuple(t.shape) != tuple(shape):
            raise ValueError(f"{name}: stored {list(t.shape)}, expected {list(shape)}")
        return t

    @classmethod
    def build(cls, cfg: DecoderConfig, qcfg: QuantConfig, seed: int = 0, device=None,
              quantize_lm_head: bool = True) -> "PackedModel":
        """The weights ``TPDecoder`` draws from ``seed``, packed once."""
        src = SeededWeights(qcfg, seed, torch.device(device or "cpu"))
        packed, tensors = {}, {"embed": src.tensor("embed", (cfg.vocab, cfg.hidden))}
        for layer in range(cfg.n_layers):
            for mat, shape in layer_shapes(cfg).items():
                packed[f"layers.{layer}.{mat}"] = src.packed(f"layers.{layer}.{mat}", shape)
        head = src.tensor("lm_head", (cfg.vocab, cfg.hidden))
        if quantize_lm_head:
            packed["lm_head"] = quantize_tensor(head, qcfg)
        else:
            tensors["lm_head"] = head
        return cls(cfg, qcfg, packed, tensors)

    def save(self, path) -> None:
        """Write to ``path`` in the ``packed_io`` format."""
        from dataclasses import asdict

        from dequant_project_b200.packed_io import save_packed
        q = self.qcfg
        save_packed(path, self.packed_weights, self.tensors,
                    meta={"decoder": asdict(self.cfg),
                          "quant": {"bits": q.bits, "group_size": q.group_size,
                                    "symmetric": q.symmetric, "layout": q.layout}})

    @classmethod
    def load(cls, path, device=None) -> "PackedModel":
        """Read a file written by ``save`` (tensors moved to ``device``)."""
        from dequant_project_b200.packed_io import load_packed
        packed, tensors, meta = load_packed(path, device)
        try:
            cfg = DecoderConfig(**meta["decoder"])
            qcfg = QuantConfig(**meta["quant"])
        except (KeyError, TypeError) as exc:
            raise ValueError(f"{path}: no decoder metadata ({exc})") from None
        return cls(cfg, qcfg, packed, tensors)


class TPDecoder:
    """This rank's shard of a packed decoder, plus its KV cache.

    ``world``/``rank``/``group`` describe the tensor-parallel process group
    (``world == 1``: no collectives). Query and KV heads split evenly over the
    ranks (both counts must divide by ``world``); the MLP's intermediate
    dimension splits on quantization-group boundaries
    (``intermediate_bounds``), the vocabulary evenly to within one row.
    ``linear_fn(x, pw)`` replaces the GEMV (tests run the host logic on the
    CPU with a dequantize-then-matmul stand-in). ``weights`` is where the full
    matrices come from: ``None`` draws them from ``seed`` and quantizes them
    (``SeededWeights``); a ``PackedModel`` (``PackedModel.load`` reads one
    from disk) supplies them already packed, so no rank quantizes anything.
    Each rank takes its shard of every full matrix. ``allreduce`` picks the
    collective after the row-parallel layers on CUDA ranks: ``"peer"`` (the
    GEMV, then the one-shot all-reduce over peer memory of ``peer_reduce``,
    run inside the residual add + RMSNorm that follows unless ``fuse_norm``
    is False; the default), ``"fused"`` (one kernel: the row-parallel GEMV exchanging
    its partial rows through peer memory, where the shape has a fused plan) or
    ``"nccl"`` (``torch.distributed.all_reduce``); CPU ranks always use the
    process group. ``close()`` releases the peer mappings.

    With ``l2_prefetch`` (CUDA ranks, packed GEMVs), the element-wise ops
    bring later GEMVs' packed weights into L2 while HBM would otherwise sit
    idle: RoPE (before the attention) the output projection and gate/up,
    the second norm the down projection, SwiGLU the next layer's QKV (the
    first norm the first layer's). ``prefetch_plan()`` lists them. With
    ``fuse_swiglu`` (CUDA, packed GEMVs with a direct-kernel plan) the gate/up
    GEMV and SwiGLU run as one kernel on gate/up rows stored interleaved by
    eights (``gu_order``; the SwiGLU's L2 prefetch is then not issued). Off by
    default: on the Llama-2-7B step it measured slower (2.36 against 2.24
    ms/token at batch 1; the prefetches compete with the running GEMV)."""

    def __init__(self, cfg: DecoderConfig, qcfg: QuantConfig, *, world: int = 1, rank: int = 0,
                 group=None, device=None, seed: int = 0, batch: int = 1, kv_len: int = 2048,
                 max_new: int = 1, quantize_lm_head: bool = True,
                 linear_fn: Callable | None = None, weights=None, allreduce: str = "peer",
                 l2_prefetch: bool = False, fuse_norm: bool = True, fuse_swiglu: bool = True):
        if cfg.n_heads % world or cfg.n_kv_heads % world:
            raise ValueError(f"{cfg.n_heads} query / {cfg.n_kv_heads} KV heads do not split "
                             f"over {world} ranks")
        if cfg.n_heads % cfg.n_kv_heads:
            raise ValueError("query heads must be a multiple of KV heads")
        self.cfg, self.qcfg = cfg, qcfg
        self.world, self.rank, self.group = world, rank, group
        self.device = torch.device(device) if device is not None else torch.device("cpu")
        self.batch, self.kv_len = batch, kv_len
        self.capacity = kv_len + max_new
        self._linear = linear_fn or _default_linear
        d = cfg.head_dim
        self.hq = cfg.n_heads // world
        self.hkv = cfg.n_kv_heads // world
        src = weights if weights is not None else SeededWeights(qcfg, seed, self.device)
        if isinstance(src, PackedModel):
            if src.cfg != cfg or src.qcfg != qcfg:
                raise ValueError("the packed model's configuration differs from cfg/qcfg")
            quantize_lm_head = "lm_head" in src.packed_weights
        shapes = layer_shapes(cfg)

        def packed(layer, mat):
            pw = src.packed(f"layers.{layer}.{mat}", shapes[mat])
            if pw.qweight.device != self.device:
                pw = PackedWeight(pw.qweight.to(self.device), pw.scales.to(self.device),
                                  None if pw.zeros is None else pw.zeros.to(self.device),
                                  pw.config, pw.shape)
            return pw

        q_bounds = [b * self.hq * d for b in range(world + 1)]
        kv_bounds = [b * self.hkv * d for b in range(world + 1)]
        self.inter_bounds = intermediate_bounds(cfg.intermediate, qcfg, world)
        self.vocab_bounds = split_bounds(cfg.vocab, world)
        self.layers = []
        for layer in range(cfg.n_layers):
            wq, wk, wv = packed(layer, "q"), packed(layer, "k"), packed(layer, "v")
            qkv = cat_rows([shard_columns(wq, world, rank, q_bounds),
                            shard_columns(wk, world, rank, kv_bounds),
                            shard_columns(wv, world, rank, kv_bounds)])
            del wq, wk, wv
            wo = packed(layer, "o")
            o, _, _ = shard_rows(wo, world, rank, q_bounds)
            del wo
            wg, wu = packed(layer, "gate"), packed(layer, "up")
            gu = cat_rows([shard_columns(wg, world, rank, self.inter_bounds),
                           shard_columns(wu, world, rank, self.inter_bounds)])
            del wg, wu
            wd = packed(layer, "down")
            down, _, _ = shard_rows(wd, world, rank, self.inter_bounds)
            del wd
            self.layers.append({"qkv": qkv, "o": o, "gu": gu, "down": down})
        self.ir = self.inter_bounds[rank + 1] - self.inter_bounds[rank]
        # Gate/up GEMV fused with SwiGLU (one kernel) where the direct kernel
        # has a plan: the packed gate/up rows are stored interleaved by eights
        # (decode_ops.gate_up_order); `gu_order` records that order.
        self.gu_order = None
        if (fuse_swiglu and self.device.type == "cuda" and self._linear is _default_linear
                and self.ir % 8 == 0):
            from dequant_project_b200.quant_linear import _format_args
            bits, gs, _, _ = _format_args(qcfg, cfg.hidden)
            if ops.gemv_swiglu_supported(batch, 2 * self.ir, cfg.hidden, bits, gs):
                order = ops.gate_up_order(self.ir).to(self.device)
                for w in self.layers:
                    gu = w["gu"]
                    w["gu"] = PackedWeight(gu.qweight[order].contiguous(),
                                           gu.scales[order].contiguous(),
                                           None if gu.zeros is None else gu.zeros[order].contiguous(),
                                           gu.config, gu.shape)
                self.gu_order = order
        self.embed = src.tensor("embed", (cfg.vocab, cfg.hidden)).to(self.device)
        lo, hi = self.vocab_bounds[rank], self.vocab_bounds[rank + 1]
        if isinstance(src, PackedModel) and quantize_lm_head:
            head = src.packed("lm_head", (cfg.vocab, cfg.hidden))
            head = PackedWeight(head.qweight.to(self.device), head.scales.to(self.device),
                                None if head.zeros is None else head.zeros.to(self.device),
                                head.config, head.shape)
            self.lm_head = shard_columns(head, world, rank, self.vocab_bounds)
        else:
            head = src.tensor("lm_head", (cfg.vocab, cfg.hidden)).to(self.device)
            if quantize_lm_head:
                self.lm_head = shard_columns(quantize_tensor(head, qcfg), world, rank,
                                             self.vocab_bounds)
            else:
                self.lm_head = head[lo:hi].contiguous()
        del head
        ones = torch.ones(cfg.hidden, dtype=torch.float16, device=self.device)
        self.attn_norm = [ones] * cfg.n_layers
        self.mlp_norm = [ones] * cfg.n_layers
        self.final_norm = ones
        self.cos, self.sin = rope_tables(d, cfg.rope_theta, self.capacity, self.device)
        self.reset_cache(seed)
        self._attn_ws = (ops.attention_workspace(batch, self.hq, self.hkv, self.capacity,
                                                 self.device)
                         if self.device.type == "cuda" else None)
        if allreduce not in ("peer", "fused", "nccl"):
            raise ValueError(f"allreduce must be 'peer', 'fused' or 'nccl', got {allreduce!r}")
        self._peer = None
        self._pf = self._prefetch_spans() if l2_prefetch else None
        self._fused = allreduce == "fused"
        # "peer": the all-reduce after a row-parallel layer runs inside the
        # residual add + RMSNorm that follows it (one kernel instead of two).
        self._norm_fused = (fuse_norm and allreduce == "peer" and world > 1
                            and self.device.type == "cuda" and cfg.hidden % 8 == 0
                            and cfg.hidden <= 8192 and not l2_prefetch)
        if world > 1 and allreduce != "nccl" and self.device.type == "cuda":
            from dequant_project_b200.peer_reduce import PeerAllReduce
            self._peer = PeerAllReduce(group, self.device, batch * cfg.hidden)

    def close(self) -> None:
        """Release the peer all-reduce's mappings (before the process group
        is destroyed); the decoder then uses the process group's all-reduce."""
        if self._peer is not None:
            self._peer.close()
            self._peer = None

    # ------------------------------------------------------------------ cache
    def reset_cache(self, seed: int = 0) -> None:
        """KV cache [batch, kv heads of this rank, capacity, head_dim] per
        layer; positions < kv_len are N(0, 1) fp16 (this rank's heads of the
        full cache, so every tensor-parallel width sees the same values)."""
        cfg, d = self.cfg, self.cfg.head_dim
        gen = torch.Generator(device=self.device)
        self.k_cache, self.v_cache = [], []
        h0 = self.rank * self.hkv
        for layer in range(cfg.n_layers):
            for which, dst in ((0, self.k_cache), (1, self.v_cache)):
                gen.manual_seed(seed * 7_919 + 2 * layer + which + 1)
                full = torch.randn((self.batch, cfg.n_kv_heads, self.kv_len, d), generator=gen,
                                   device=self.device, dtype=torch.float32).to(torch.float16)
                c = torch.zeros((self.batch, self.hkv, self.capacity, d), dtype=torch.float16,
                                device=self.device)
                c[:, :, :self.kv_len] = full[:, h0:h0 + self.hkv]
                dst.append(c)

    def prefetch_plan(self) -> dict:
        """{(layer, op): [matrix names]} of the step's L2 prefetches, op one
        of "norm1", "rope", "norm2", "silu"."""
        plan = {}
        for layer in range(self.cfg.n_layers):
            if layer == 0:
                plan[(0, "norm1")] = [(0, "qkv")]
            plan[(layer, "rope")] = [(layer, "o"), (layer, "gu")]
            plan[(layer, "norm2")] = [(layer, "down")]
            if layer + 1 < self.cfg.n_layers:
                plan[(layer, "silu")] = [(layer + 1, "qkv")]
        return plan

    def _prefetch_spans(self) -> dict | None:
        if self.device.type != "cuda" or self._linear is not _default_linear:
            return None
        return {key: ops.l2_spans([self.layers[lay][mat] for lay, mat in mats])
                for key, mats in self.prefetch_plan().items()}

    def _prefetch(self, layer: int, op: str):
        return None if self._pf is None else self._pf.get((layer, op))

    # -------------------------------------------------------------- forward
    def _all_reduce(self, t: torch.Tensor) -> torch.Tensor:
        if self._peer is not None:
            return self._peer(t)
        if self.world > 1:
            import torch.distributed as dist
            dist.all_reduce(t, op=dist.ReduceOp.SUM, group=self.group)
        return t

    def _row_parallel(self, x: torch.Tensor, pw: PackedWeight) -> tuple:
        """A row-parallel layer: (output, reduced). With the fused GEMV +
        peer all-reduce (``allreduce="fused"``) one kernel where the shape has
        a fused plan; with the peer collective ("peer") this rank's partial
        output, unreduced (``reduced`` False: the norm that follows reduces
        it); otherwise this rank's GEMV and the all-reduce."""
        if self._peer is not None and self._fused and self._linear is _default_linear:
            return self._peer.gemv(x, pw), True
        if self._peer is not None and self._norm_fused:
            return self._linear(x, pw), False
        return self._all_reduce(self._linear(x, pw)), True

    def _add_norm(self, h, delta, weight, reduced: bool, prefetch=None) -> torch.Tensor:
        """Residual add + RMSNorm; a delta that is still a row-parallel
        layer's unreduced partial is all-reduced by the same kernel."""
        if delta is not None and not reduced:
            return self._peer.add_rms_norm(delta, h, weight, self.cfg.eps)
        return ops.add_rms_norm(h, delta, weight, self.cfg.eps, prefetch)

    def _lm_head(self, x: torch.Tensor) -> torch.Tensor:
        if isinstance(self.lm_head, PackedWeight):
            return self._linear(x, self.lm_head)
        return F.linear(x, self.lm_head)

    def step(self, tokens: torch.Tensor, pos: int) -> torch.Tensor:
        """One decode step: tokens [batch] int64 at position ``pos`` (their K/V
        go to cache slot ``pos``, attention covers positions 0..pos). Returns
        the full logits [batch, vocab] fp16 on every rank.

        Per layer five kernels surround the three packed GEMVs and the two
        all-reduces: residual add + RMSNorm (the residual of the previous
        block folded in), RoPE + KV append, attention, residual add + RMSNorm,
        SwiGLU."""
        cfg, d = self.cfg, self.cfg.head_dim
        if not 0 <= pos < self.capacity:
            raise ValueError(f"position {pos} outside the cache (capacity {self.capacity})")
        m = tokens.shape[0]
        if m != self.batch:
            raise ValueError(f"expected {self.batch} tokens, got {m}")
        h = self.embed[tokens]
        cos, sin = self.cos[pos], self.sin[pos]
        nq = self.hq * d
        pending, reduced = None, True
        for layer, w in enumerate(self.layers):
            x = self._add_norm(h, pending, self.attn_norm[layer], reduced,
                               self._prefetch(layer, "norm1"))
            qkv = self._linear(x, w["qkv"])
            kc, vc = self.k_cache[layer], self.v_cache[layer]
            q = ops.rope_kv_append(qkv, cos, sin, kc, vc, pos, self.hq, self.hkv,
                                   self._prefetch(layer, "rope"))
            a = ops.attention(q, kc, vc, pos + 1, self._attn_ws)
            o, o_reduced = self._row_parallel(a.reshape(m, nq), w["o"])
            x = self._add_norm(h, o, self.mlp_norm[layer], o_reduced,
                               self._prefetch(layer, "norm2"))
            if self.gu_order is not None:
                act = ops.gemv_swiglu(x, w["gu"])
            else:
                act = ops.silu_mul(self._linear(x, w["gu"]), self._prefetch(layer, "silu"))
            pending, reduced = self._row_parallel(act, w["down"])
        x = self._add_norm(h, pending, self.final_norm, reduced)
        logits = self._lm_head(x)
        if self.world == 1:
            return logits
        import torch.distributed as dist
        width = max(b - a for a, b in zip(self.vocab_bounds[:-1], self.vocab_bounds[1:]))
        padded = logits.new_zeros((m, width))
        padded[:, :logits.shape[1]] = logits
        parts = [torch.empty_like(padded) for _ in range(self.world)]
        dist.all_gather(parts, padded, group=self.group)
        return torch.cat([p[:, :b - a] for p, a, b in
                          zip(parts, self.vocab_bounds[:-1], self.vocab_bounds[1:])], dim=1)

    def generate(self, tokens: torch.Tensor, steps: int, start: int | None = None) -> torch.Tensor:
        """Greedy decode: feed ``tokens`` [batch] at position ``start`` (default
        ``kv_len``), then each step's argmax, ``steps`` times. Returns the
        generated ids [batch, steps] (identical on every rank: the logits are
        all-gathered before the argmax). Needs ``start + steps <= capacity``."""
        pos = self.kv_len if start is None else start
        if pos + steps > self.capacity:
            raise ValueError(f"{steps} steps from position {pos} exceed the cache capacity "
                             f"{self.capacity}")
        out = []
        cur = tokens
        for t in range(steps):
            cur = self.step(cur, pos + t).argmax(dim=-1)
            out.append(cur)
        return torch.stack(out, dim=1)

    def packed_bytes(self) -> int:
        """Bytes of this rank's packed weights (layers and LM head)."""
        n = sum(pw.nbytes for w in self.layers for pw in w.values())
        head = self.lm_head
        return n + (head.nbytes if isinstance(head, PackedWeight) else head.numel() * 2)

    def step_bytes(self, pos: int) -> dict:
        """Bytes one step at ``pos`` must move on this rank (the terms of the
        reference's decode byte model, dequant/byte_model.py:179-251, for this
        rank's shard): packed weights and LM head, the KV cache read for
        positions 0..pos and the new slot written, the embedding row, norm
        weights; activations (a few KB) are left out."""
        cfg, d = self.cfg, self.cfg.head_dim
        kv_read = cfg.n_layers * 2 * self.batch * self.hkv * (pos + 1) * d * 2
        kv_write = cfg.n_layers * 2 * self.batch * self.hkv * d * 2
        out = {"weights": self.packed_bytes(), "kv_cache": kv_read + kv_write,
               "embedding": self.batch * cfg.hidden * 2,
               "norms": (2 * cfg.n_layers + 1) * cfg.hidden * 2}
        out["total"] = sum(out.values())
        return out


class DecodeGraph:
    """One decode step at a fixed position, captured in a CUDA graph on this
    rank (GEMVs, attention and the collectives). ``replay()`` reruns it on the
    current contents of ``tokens``; ``logits`` holds the output."""

    def __init__(self, dec: TPDecoder, pos: int, warmup: int = 2):
        self.dec, self.pos = dec, pos
        self.tokens = torch.zeros(dec.batch, dtype=torch.int64, device=dec.device)
        self.stream = torch.cuda.Stream(device=dec.device)
        self.stream.wait_stream(torch.cuda.current_stream(dec.device))
        with torch.cuda.stream(self.stream):
            for _ in range(warmup):
                dec.step(self.tokens, pos)
        self.stream.synchronize()
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph, stream=self.stream):
            self.logits = dec.step(self.tokens, pos)
        self.stream.synchronize()

    def replay(self) -> torch.Tensor:
        self.graph.replay()
        return self.logits

    def release(self) -> None:
        """Drop the graph (before the process group is destroyed)."""
        self.graph.reset()
        self.graph = None
