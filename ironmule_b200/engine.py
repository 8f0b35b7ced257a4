"""The B200 speculative-decoding engine: 4-bit Qwen3 / Gemma-3 shaped models on libimspec kernels, a paged KV
cache, and the draft -> verify -> accept round captured as one CUDA graph.

This is the device counterpart of the reference's engines' step loops (IronMule ironmule/ggml_engine.py:1155-1343,
ironmule/runtime.py:702-776, ironmule/dense_plan.py:488-529): the same round -- draft k tokens with the small
model, verify them with the target in one multi-row forward, keep the agreed prefix plus the target's own
token, roll the KV back -- with the argmax, the acceptance and the bookkeeping on the device.

Layout in HBM per model: 4-bit weights (MLX affine, group 64) per layer -- qkv packed [q; k; v] rows, o,
gate/up interleaved in 16-row blocks (gate rows then the matching up rows, so one qGEMM CTA holds both halves
of the SwiGLU), down -- plus bf16 norm weights; the tied 4-bit embedding doubles as the LM head. KV caches are
[layers][pages][Hkv][16][D] bf16 with a page table per sequence slot.

Every projection is also held repacked for the packed qGEMM (`kernels.Packed`: 1152-byte units of 32 rows x 64
inputs in MMA-fragment order), which is what the forward reads.

Forward of M rows (any mix of sequences), five launches per layer (seven for Gemma-3, whose attention and MLP
outputs get their own RMSNorm before the residual add: o / down store, then im_rmsnorm_residual): embed (+ each row's sum of squares) -> per
layer [qkv qGEMM with the input RMSNorm fused into its prologue, paged attention with the q/k norm + RoPE +
KV write fused into it, o qGEMM + residual (+ per-tile sums of squares of the new h), gate/up qGEMM with the post-attention RMSNorm
fused + SwiGLU, down qGEMM + residual (+ sums of squares)] -> head qGEMM with the final RMSNorm fused, over the
leading rows that need logits. Every kernel is row-invariant (no arithmetic depends on M or on the other rows),
so a verify row's logits equal those of a one-row decode bit for bit, and speculation never changes a greedy
answer.
"""
from __future__ import annotations

import dataclasses
import math
from dataclasses import dataclass, field

import torch

from . import kernels
from .kvpool import PAGE, PagePool  # PAGE: KV slots per cache page

MAX_QGEMM_ROWS = 320   # rows of one forward (the packed qGEMM takes them in chunks of 32)
MAX_SEQ_ROWS = 32      # rows of one sequence in one forward through the fused attention
PREFILL_SEQ_ROWS = 256  # rows of one sequence in one prefill forward (above 32: q/k norm + RoPE + KV write, then
                        # the paged attention, as two kernels)
PARK_PAGES = 3         # pages an idle decoder slot writes (positions 0 .. 2 + MAX_SEQ_ROWS)


@dataclass(frozen=True)
class ModelConfig:
    name: str
    hidden: int
    layers: int
    heads: int
    kv_heads: int
    head_dim: int
    inter: int
    vocab: int
    rope_theta: float = 1_000_000.0
    eps: float = 1e-6
    family: str = "qwen3"          # "qwen3" (SwiGLU, w-norms) or "gemma3" (GeGLU, (1+w)-norms, post-norms)
    sliding_window: int = 0         # gemma3: local layers see the last `sliding_window` slots
    global_every: int = 0           # gemma3: layer i is global when (i + 1) % global_every == 0
    rope_local_theta: float = 10_000.0
    query_scale: float = 0.0        # attention scale; 0 -> head_dim ** -0.5
    rope_scale: float = 1.0         # linear RoPE scaling of the global layers (positions / rope_scale)

    @property
    def qkv_rows(self) -> int:
        return (self.heads + 2 * self.kv_heads) * self.head_dim

    @property
    def scale(self) -> float:
        return self.query_scale or self.head_dim ** -0.5

    def params(self) -> int:
        per_layer = (self.hidden * self.qkv_rows + self.heads * self.head_dim * self.hidden
                     + 3 * self.hidden * self.inter)
        return self.layers * per_layer + self.vocab * self.hidden

    def weight_bytes(self) -> int:
        """Bytes of 4-bit weights (0.5 B per weight + 4 B of scale and bias per 64) read by one forward pass."""
        return self.params() * 9 // 16

    def kv_bytes_per_token(self) -> int:
        return self.layers * 2 * self.kv_heads * self.head_dim * 2

    def is_global(self, layer: int) -> bool:
        return self.family != "gemma3" or self.global_every == 0 or (layer + 1) % self.global_every == 0


PRESETS = {
    # BASELINE configs 2/3: Qwen3-4B target and Qwen3-0.6B draft (tied embeddings, vocab 151936)
    "qwen3-4b": ModelConfig("qwen3-4b", 2560, 36, 32, 8, 128, 9728, 151936),
    "qwen3-0.6b": ModelConfig("qwen3-0.6b", 1024, 28, 16, 8, 128, 3072, 151936),
    # BASELINE config 4 / 5a: Gemma-3 12B and 27B (sliding window 1024 on 5 of 6 layers)
    "gemma3-12b": ModelConfig("gemma3-12b", 3840, 48, 16, 8, 256, 15360, 262144, family="gemma3",
                              sliding_window=1024, global_every=6, query_scale=256 ** -0.5),
    "gemma3-27b": ModelConfig("gemma3-27b", 5376, 62, 32, 16, 128, 21504, 262144, family="gemma3",
                              sliding_window=1024, global_every=6, query_scale=168 ** -0.5),
    # a Gemma-3-1B-shaped draft for the Gemma-3 tree workload (the configuration leaves the draft open)
    "gemma3-1b": ModelConfig("gemma3-1b", 1152, 26, 4, 1, 256, 6912, 262144, family="gemma3", sliding_window=512,
                             global_every=6, query_scale=256 ** -0.5),
    # small shapes for tests
    "tiny-target": ModelConfig("tiny-target", 256, 2, 4, 2, 128, 512, 1000),
    "tiny-draft": ModelConfig("tiny-draft", 128, 2, 2, 1, 128, 256, 1000),
    "tiny-gemma": ModelConfig("tiny-gemma", 256, 3, 4, 2, 128, 512, 1000, family="gemma3", sliding_window=16,
                              global_every=3, query_scale=128 ** -0.5),
}


@dataclass
class Linear4:
    """One 4-bit projection on the device: MLX layout (w, s, b) and the packed copy the forward reads."""
    w: torch.Tensor
    s: torch.Tensor
    b: torch.Tensor
    p: kernels.Packed | None = None

    @property
    def n(self) -> int:
        return int(self.w.shape[0])

    @property
    def k(self) -> int:
        return int(self.w.shape[1]) * 8


@dataclass
class Layer:
    qkv: Linear4
    o: Linear4
    gate_up: Linear4
    down: Linear4
    in_norm: torch.Tensor
    post_norm: torch.Tensor      # the norm before the MLP (Gemma-3: pre_feedforward_layernorm)
    q_norm: torch.Tensor
    k_norm: torch.Tensor
    post_attn_norm: torch.Tensor | None = None  # Gemma-3: on the attention output before its residual add
    post_ff_norm: torch.Tensor | None = None    # Gemma-3: on the MLP output before its residual add


def interleave_gate_up(gate: torch.Tensor, up: torch.Tensor) -> torch.Tensor:
    """[I, K] gate and up -> [2I, K] in 16-row blocks: gate[16j:16j+16], up[16j:16j+16], ..."""
    inter, k = gate.shape
    if inter % 16:
        raise ValueError("intermediate size must be a multiple of 16")
    return torch.stack([gate.view(inter // 16, 16, k), up.view(inter // 16, 16, k)], dim=1).reshape(2 * inter, k)


def tp_shard(cfg: ModelConfig, tp: int, r: int) -> dict[str, tuple[int, int]]:
    """Rank r's slices of a tp-way tensor-parallel model, as [start, end) ranges of the full matrices: rows of
    the q, k and v blocks of qkv, columns of o (= its q heads' outputs), rows of gate and of up, columns of down,
    rows of the tied embedding used as the head."""
    d = cfg.head_dim
    hq, hkv, il, vl = cfg.heads // tp, cfg.kv_heads // tp, cfg.inter // tp, cfg.vocab // tp
    q0, k0, v0 = r * hq * d, cfg.heads * d + r * hkv * d, (cfg.heads + cfg.kv_heads) * d + r * hkv * d
    return {"q": (q0, q0 + hq * d), "k": (k0, k0 + hkv * d), "v": (v0, v0 + hkv * d),
            "o_cols": (r * hq * d, (r + 1) * hq * d), "inter": (r * il, (r + 1) * il),
            "vocab": (r * vl, (r + 1) * vl)}


@dataclass
class RowMeta:
    """Device metadata for a forward of M rows: token ids (with a stride), slot / position / sequence per row,
    sequence row offsets [B+1]; static host facts for the launch geometry."""
    tokens: torch.Tensor
    token_stride: int
    pos: torch.Tensor
    seq: torch.Tensor  # sequence group per row (an index into seq_rows, and into seq_slot when given)
    seq_rows: torch.Tensor
    rows: int
    max_rows_per_seq: int
    seq_slot: torch.Tensor | None = None  # page-table row per sequence group (None: group b is slot b)
    slot: torch.Tensor | None = None      # KV slot per row when it differs from the position (draft trees)
    tree_mask: torch.Tensor | None = None  # int64 per row: ancestor bits over the tree slots
    tree_base: torch.Tensor | None = None  # int32 per sequence group: the first tree slot


class QuantModel:
    """A random-init 4-bit model resident on one GPU, with its paged KV cache and preallocated activations.

    Tensor parallelism (tp > 1, one process per GPU, `group` a NCCL process group of tp ranks): rank r holds
    heads [r Hq/tp, (r+1) Hq/tp) of q and of k/v (column shards of qkv), the matching columns of o (a row
    shard along K), rows [r I/tp, (r+1) I/tp) of gate and up (column shards, still 16-row interleaved) and the
    matching columns of down, its kv heads' cache, and vocabulary rows [r V/tp, (r+1) V/tp) of the tied head;
    the embedding table (for the gather) and the norms are replicated. The shards are cut from the same seeded
    full matrices a tp = 1 model of the same seed holds, and 64-element groups never straddle a cut, so the
    quantised shards are slices of the tp = 1 model's weights. Forward: o and down store their partial sums,
    an all-reduce (sum, bf16) adds them, then the (post-)norm + residual kernel; the head's vocabulary slices are
    all-gathered into full logits, so acceptance sees the whole vocabulary on every rank (BASELINE config 5a;
    the reference has no tensor parallelism).
    """

    def __init__(self, cfg: ModelConfig, device: torch.device | str = "cuda", *, seed: int = 0,
                 sigma: float = 0.02, max_seqs: int = 1, max_ctx: int = 1024, max_rows: int = 32,
                 max_logit_rows: int = 32, keys_per_split: int | None = None, tp: int = 1, rank: int = 0, group=None,
                 weights: dict | None = None):
        self.cfg = cfg
        if tp > 1 and (cfg.heads % tp or cfg.kv_heads % tp or cfg.inter % (64 * tp) or (cfg.inter // tp) % 16
                       or cfg.vocab % tp or (cfg.heads * cfg.head_dim // tp) % 64):
            raise ValueError(f"{cfg.name} does not split {tp} ways (heads, kv heads, 64-groups of K, vocabulary)")
        self.tp, self.rank, self.group = tp, rank, group
        # the rank's shapes: its heads and its slice of the intermediate size (the full model when tp == 1)
        self.lc = dataclasses.replace(cfg, heads=cfg.heads // tp, kv_heads=cfg.kv_heads // tp, inter=cfg.inter // tp)
        self.device = torch.device(device)
        self.max_seqs, self.max_rows, self.max_logit_rows = max_seqs, max_rows, max_logit_rows
        self.pages_per_seq = -(-max_ctx // PAGE)
        self.max_ctx = self.pages_per_seq * PAGE
        # attention keys per split, fixed per model (so every forward of the model splits a row's keys alike):
        # 128 for one sequence (enough splits to spread it over the GPU), 256 for batches (fewer partials to merge;
        # measured on B200: config-3 verify attention 166 vs 205 us, config-2 draft pass 11.3 vs 16.3 us at 256)
        self.keys_per_split = keys_per_split or (128 if max_seqs == 1 else 256)
        if weights is None:
            gen = torch.Generator(device=self.device).manual_seed(seed)
            self._build_weights(gen, sigma)
        else:  # a checkpoint's 4-bit tensors under MLX names (ironmule_b200.checkpoint)
            from .checkpoint import assign_weights
            assign_weights(self, weights)
        self._build_rope()
        self._build_cache()
        self._build_buffers()

    # ---- weights ----------------------------------------------------------------------------------------
    def _rand(self, gen, n, k, sigma) -> torch.Tensor:
        return (torch.randn((n, k), generator=gen, device=self.device) * sigma).to(torch.bfloat16)

    def _lin(self, w: torch.Tensor) -> Linear4:
        wq, s, b = kernels.quantize(w.contiguous())
        return Linear4(wq, s, b, kernels.Packed(wq, s, b))

    def _norm(self, gen, n) -> torch.Tensor:
        base = 0.0 if self.cfg.family == "gemma3" else 1.0
        return (base + 0.02 * torch.randn((n,), generator=gen, device=self.device)).to(torch.bfloat16)

    def _build_weights(self, gen, sigma) -> None:
        c, tp = self.cfg, self.tp
        sh = tp_shard(c, tp, self.rank)
        cut = lambda a, key: a[slice(*sh[key])]  # noqa: E731
        table = self._rand(gen, c.vocab, c.hidden, sigma)
        if tp == 1:
            self.embed = self._lin(table)
            self.head = self.embed
        else:
            wq, s, b = kernels.quantize(table.contiguous())
            self.embed = Linear4(wq, s, b)  # the gather reads the whole table; the head is this rank's slice
            self.head = self._lin(cut(table, "vocab"))
        del table
        self.layers: list[Layer] = []
        for _ in range(c.layers):
            qkv_full = self._rand(gen, c.qkv_rows, c.hidden, sigma)
            if tp > 1:
                qkv_full = torch.cat([cut(qkv_full, "q"), cut(qkv_full, "k"), cut(qkv_full, "v")])
            qkv = self._lin(qkv_full)
            o_full = self._rand(gen, c.hidden, c.heads * c.head_dim, sigma)
            o = self._lin(o_full[:, slice(*sh["o_cols"])] if tp > 1 else o_full)
            gate, up = self._rand(gen, c.inter, c.hidden, sigma), self._rand(gen, c.inter, c.hidden, sigma)
            if tp > 1:
                gate, up = cut(gate, "inter"), cut(up, "inter")
            gate_up = self._lin(interleave_gate_up(gate.contiguous(), up.contiguous()))
            del gate, up, qkv_full, o_full
            down_full = self._rand(gen, c.hidden, c.inter, sigma)
            down = self._lin(down_full[:, slice(*sh["inter"])] if tp > 1 else down_full)
            del down_full
            layer = Layer(qkv, o, gate_up, down, self._norm(gen, c.hidden), self._norm(gen, c.hidden),
                          self._norm(gen, c.head_dim), self._norm(gen, c.head_dim))
            if c.family == "gemma3":
                layer.post_attn_norm, layer.post_ff_norm = self._norm(gen, c.hidden), self._norm(gen, c.hidden)
            self.layers.append(layer)
        self.final_norm = self._norm(gen, c.hidden)

    def _build_rope(self) -> None:
        c, d = self.cfg, self.cfg.head_dim
        idx = torch.arange(0, d // 2, dtype=torch.float64)
        self.inv_freq = (c.rope_theta ** (-2.0 * idx / d) / c.rope_scale).to(torch.float32).to(self.device)
        self.inv_freq_local = (c.rope_local_theta ** (-2.0 * idx / d)).to(torch.float32).to(self.device)

    # ---- cache and buffers ------------------------------------------------------------------------------
    def _build_cache(self) -> None:
        c = self.lc
        pages = self.max_seqs * self.pages_per_seq
        shape = (c.layers, pages, c.kv_heads, PAGE, c.head_dim)
        self.k_cache = torch.zeros(shape, dtype=torch.bfloat16, device=self.device)
        self.v_cache = torch.zeros(shape, dtype=torch.bfloat16, device=self.device)
        # a fixed page range per sequence slot; the table is what the kernels read
        self.page_table = torch.arange(pages, dtype=torch.int32, device=self.device).view(self.max_seqs, -1)

    def _build_buffers(self) -> None:
        c, r, dev = self.lc, self.max_rows, self.device
        bf = torch.bfloat16
        self.h = torch.zeros((r, c.hidden), dtype=bf, device=dev)
        # row sums of squares of h for the fused RMSNorms: one part from the embedding, one per 32-row tile
        # of the hidden dimension from the residual epilogues
        self.h_tiles = -(-c.hidden // 32)
        self.sq_ld = -(-min(r, MAX_QGEMM_ROWS) // 32) * 32  # row stride of the sums-of-squares buffers
        self.sq_embed = torch.zeros((self.sq_ld,), dtype=torch.float32, device=dev)
        self.sq_attn = torch.zeros((self.h_tiles, self.sq_ld), dtype=torch.float32, device=dev)
        self.sq_mlp = torch.zeros((self.h_tiles, self.sq_ld), dtype=torch.float32, device=dev)
        self.qkv = torch.zeros((r, c.qkv_rows), dtype=bf, device=dev)
        self.attn = torch.zeros((r, c.heads * c.head_dim), dtype=bf, device=dev)  # [M, Hq, D] packed
        self.act = torch.zeros((r, c.inter), dtype=bf, device=dev)
        self.y = torch.zeros((r, c.hidden), dtype=bf, device=dev)  # Gemma-3: projection output before its norm
        self.logits = torch.zeros((self.max_logit_rows, c.vocab), dtype=bf, device=dev)
        if self.tp > 1:  # this rank's vocabulary slice, and the all-gather target [tp][rows][V/tp]
            vl = c.vocab // self.tp
            self.logits_local = torch.zeros((self.max_logit_rows, vl), dtype=bf, device=dev)
            self.logits_gather = torch.zeros((self.tp * self.max_logit_rows * vl,), dtype=bf, device=dev)
        # scratch: one buffer per kernel family, sized for the largest call this model makes
        q_need = max(kernels.qgemm_packed_workspace_bytes(min(r, MAX_QGEMM_ROWS), n, k)
                     for n, k in self._gemm_shapes())
        head_need = kernels.qgemm_packed_workspace_bytes(self.max_logit_rows, c.vocab // self.tp, c.hidden)
        self.ws_gemm = kernels.workspace(max(q_need, head_need), dev)
        a_need = max(kernels.attention_workspace_bytes(self.max_seqs, rows, c.heads, c.kv_heads, c.head_dim,
                                                       self.max_ctx, self.keys_per_split)
                     for rows in (1, 8, min(r, MAX_SEQ_ROWS), min(r, PREFILL_SEQ_ROWS)))
        self.ws_attn = kernels.workspace(a_need, dev)
        # the roped queries of forwards with more rows per sequence than the fused attention takes (prefill)
        self.q_wide = torch.zeros((r, c.heads * c.head_dim), dtype=bf, device=dev) if r > MAX_SEQ_ROWS else None
        # forwards of at most this many rows merge the attention's splits in the o-projection's prologue (not with
        # tensor parallelism or Gemma-3's post-attention norm, whose o-projections have no residual epilogue)
        self.o_merge_rows = (kernels.qgemm_packed_attn_rows(c.hidden, c.heads * c.head_dim)
                             if self.tp == 1 and c.family != "gemma3" else 0)
        self.ws_argmax = kernels.workspace(kernels.argmax_workspace_bytes(self.max_logit_rows, c.vocab), dev)

    def _gemm_shapes(self):
        c = self.lc
        return [(c.qkv_rows, c.hidden), (c.hidden, c.heads * c.head_dim), (2 * c.inter, c.hidden),
                (c.hidden, c.inter)]

    # ---- forward ------------------------------------------------------------------------------------------
    def forward(self, meta: RowMeta, max_kv_len: int, logit_rows: int = 0,
                trace: list | None = None) -> torch.Tensor | None:
        """Run M = meta.rows rows through the model, writing their K/V at their slots; the logits of the first
        `logit_rows` rows land in self.logits[:logit_rows] (returned; None when logit_rows is 0). With a `trace`
        list, one dict per layer is appended holding copies of the rows at each op boundary -- "h_in" (the layer's
        input), "qkv", "attn", "h_mid" (after the attention residual) and "act" (after the gated MLP activation) --
        and a last dict with the final hidden rows as "h_in" (the parity tests feed each op's device input to the
        CPU restatement of that op); never inside a captured graph."""
        c, m = self.lc, meta.rows
        if m > min(self.max_rows, MAX_QGEMM_ROWS):
            raise ValueError(f"{m} rows exceed this model's per-forward limit")
        if logit_rows > min(m, self.max_logit_rows):
            raise ValueError(f"{logit_rows} logit rows exceed the rows or this model's logit buffer")
        gemma = c.family == "gemma3"
        mult = math.sqrt(c.hidden) if gemma else 1.0
        h, ws = self.h, self.ws_gemm
        kernels.embed(meta.tokens, self.embed.w, self.embed.s, self.embed.b, mult=mult, out=h, rows=m,
                      stride=meta.token_stride, out_sq=self.sq_embed)
        sq, parts = self.sq_embed, 1
        row_page = None  # page-table row of every row, for the two-kernel attention of wide prefill chunks
        if meta.max_rows_per_seq > MAX_SEQ_ROWS:
            if self.q_wide is None or m > self.q_wide.shape[0]:
                raise ValueError(f"{meta.max_rows_per_seq} rows of one sequence exceed this model's rows")
            row_page = meta.seq if meta.seq_slot is None else meta.seq_slot[meta.seq.long()]
        def tr(key: str, t: torch.Tensor) -> None:
            if trace is not None:
                trace[-1][key] = t[:m].clone()

        for li, layer in enumerate(self.layers):
            if trace is not None:
                trace.append({"h_in": h[:m].clone()})
            kernels.qgemm_packed(h, layer.qkv.p, out=self.qkv, rows=m, norm_sq=sq, norm_parts=parts,
                                 norm_weight=layer.in_norm, eps=c.eps, gemma_norm=gemma, sq_ld=self.sq_ld, ws=ws)
            tr("qkv", self.qkv)
            glob = c.is_global(li)
            row_slot = meta.pos if meta.slot is None else meta.slot
            # few rows: the attention leaves its split partials for the o-projection's prologue to merge (same
            # bits; the per-op trace keeps the attention output, so it takes the unmerged route)
            merge_in_o = m <= self.o_merge_rows and trace is None
            inv_freq = self.inv_freq if glob else self.inv_freq_local
            window = 0 if glob else c.sliding_window
            if meta.max_rows_per_seq > MAX_SEQ_ROWS:  # prefill chunks beyond the fused attention's rows
                q = kernels.qk_norm_rope_kv(self.qkv, layer.q_norm, layer.k_norm, inv_freq, meta.pos, row_slot, row_page,
                                            self.page_table, c.heads, c.kv_heads, c.head_dim, c.eps, self.k_cache[li],
                                            self.v_cache[li], gemma=gemma, q_out=self.q_wide, rows=m)
                kernels.attention(q.view(-1, c.heads, c.head_dim), self.k_cache[li], self.v_cache[li], self.page_table,
                                  meta.seq_rows, row_slot, max_rows_per_seq=meta.max_rows_per_seq,
                                  max_kv_len=max_kv_len, scale=c.scale, keys_per_split=self.keys_per_split,
                                  window=window, tree_mask=meta.tree_mask, tree_base=meta.tree_base, out=self.attn,
                                  rows=m, ws=self.ws_attn, seq_slot=meta.seq_slot)
            else:
                kernels.attention_qkv(self.qkv, layer.q_norm, layer.k_norm, inv_freq, meta.pos, self.k_cache[li],
                                      self.v_cache[li], self.page_table, meta.seq_rows, row_slot,
                                      tree_mask=meta.tree_mask, tree_base=meta.tree_base, hq=c.heads, hkv=c.kv_heads,
                                      d=c.head_dim, eps=c.eps, gemma=gemma, max_rows_per_seq=meta.max_rows_per_seq,
                                      max_kv_len=max_kv_len, scale=c.scale, keys_per_split=self.keys_per_split,
                                      window=window, out=self.attn, rows=m, ws=self.ws_attn, seq_slot=meta.seq_slot,
                                      defer=merge_in_o)
            if merge_in_o:
                kernels.qgemm_packed_attn(self.ws_attn, layer.o.p, meta.seq_rows, row_slot, residual=h, out=h, rows=m,
                                          max_rows_per_seq=meta.max_rows_per_seq, hq=c.heads, hkv=c.kv_heads,
                                          d=c.head_dim, max_kv_len=max_kv_len, keys_per_split=self.keys_per_split,
                                          out_sq=self.sq_attn, sq_ld=self.sq_ld, ws=ws)
            tr("attn", self.attn)
            if self.tp > 1:  # partial sums of the row-sharded o and down, all-reduced before the residual add
                kernels.qgemm_packed(self.attn, layer.o.p, out=self.y, rows=m, sq_ld=self.sq_ld, ws=ws)
                self._all_reduce(self.y[:m])
                kernels.rmsnorm_residual(self.y, layer.post_attn_norm, h, c.eps, gemma=gemma, rows=m,
                                         out_sq=self.sq_attn)
                kernels.qgemm_packed(h, layer.gate_up.p, epilogue="geglu" if gemma else "swiglu", out=self.act,
                                     rows=m, norm_sq=self.sq_attn, norm_parts=1, norm_weight=layer.post_norm,
                                     eps=c.eps, gemma_norm=gemma, sq_ld=self.sq_ld, ws=ws)
                kernels.qgemm_packed(self.act, layer.down.p, out=self.y, rows=m, sq_ld=self.sq_ld, ws=ws)
                self._all_reduce(self.y[:m])
                kernels.rmsnorm_residual(self.y, layer.post_ff_norm, h, c.eps, gemma=gemma, rows=m, out_sq=self.sq_mlp)
                sq, parts = self.sq_mlp, 1
                continue
            if gemma:  # Gemma-3: output norms before each residual add; one sum-of-squares part per row
                kernels.qgemm_packed(self.attn, layer.o.p, out=self.y, rows=m, sq_ld=self.sq_ld, ws=ws)
                kernels.rmsnorm_residual(self.y, layer.post_attn_norm, h, c.eps, gemma=True, rows=m,
                                         out_sq=self.sq_attn)
                tr("h_mid", h)
                kernels.qgemm_packed(h, layer.gate_up.p, epilogue="geglu", out=self.act, rows=m, norm_sq=self.sq_attn,
                                     norm_parts=1, norm_weight=layer.post_norm, eps=c.eps, gemma_norm=True, sq_ld=self.sq_ld, ws=ws)
                tr("act", self.act)
                kernels.qgemm_packed(self.act, layer.down.p, out=self.y, rows=m, sq_ld=self.sq_ld, ws=ws)
                kernels.rmsnorm_residual(self.y, layer.post_ff_norm, h, c.eps, gemma=True, rows=m,
                                         out_sq=self.sq_mlp)
                sq, parts = self.sq_mlp, 1
                continue
            if not merge_in_o:
                kernels.qgemm_packed(self.attn, layer.o.p, epilogue="residual", residual=h, out=h, rows=m,
                                     out_sq=self.sq_attn, sq_ld=self.sq_ld, ws=ws)
            tr("h_mid", h)
            kernels.qgemm_packed(h, layer.gate_up.p, epilogue="swiglu", out=self.act, rows=m,
                                 norm_sq=self.sq_attn, norm_parts=self.h_tiles, norm_weight=layer.post_norm,
                                 eps=c.eps, gemma_norm=gemma, sq_ld=self.sq_ld, ws=ws)
            tr("act", self.act)
            kernels.qgemm_packed(self.act, layer.down.p, epilogue="residual", residual=h, out=h, rows=m,
                                 out_sq=self.sq_mlp, sq_ld=self.sq_ld, ws=ws)
            sq, parts = self.sq_mlp, self.h_tiles
        if trace is not None:
            trace.append({"h_in": h[:m].clone()})
        if not logit_rows:
            return None
        if self.tp == 1:
            kernels.qgemm_packed(h, self.head.p, out=self.logits, rows=logit_rows, norm_sq=sq, norm_parts=parts,
                                 norm_weight=self.final_norm, eps=c.eps, gemma_norm=gemma, sq_ld=self.sq_ld, ws=ws)
            return self.logits[:logit_rows]
        lr, vl = logit_rows, c.vocab // self.tp
        kernels.qgemm_packed(h, self.head.p, out=self.logits_local, rows=lr, norm_sq=sq, norm_parts=parts,
                             norm_weight=self.final_norm, eps=c.eps, gemma_norm=gemma, sq_ld=self.sq_ld, ws=ws)
        import torch.distributed as dist
        gathered = self.logits_gather[:self.tp * lr * vl]
        with self._timed_collective():
            dist.all_gather_into_tensor(gathered, self.logits_local[:lr], group=self.group)
        self.logits[:lr].view(lr, self.tp, vl).copy_(gathered.view(self.tp, lr, vl).permute(1, 0, 2))
        return self.logits[:lr]

    def _all_reduce(self, t: torch.Tensor) -> None:
        import torch.distributed as dist
        with self._timed_collective():
            dist.all_reduce(t, op=dist.ReduceOp.SUM, group=self.group)

    def _timed_collective(self):
        """CUDA events around a collective when `collective_events` is a list (an eager, measured forward): the
        tensor-parallel bench sums their durations into the collectives' share of a round."""
        import contextlib

        events = getattr(self, "collective_events", None)
        if events is None:
            return contextlib.nullcontext()

        @contextlib.contextmanager
        def timed():
            start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            start.record()
            yield
            end.record()
            events.append((start, end))

        return timed()

    # ---- eager helpers (prefill, plain decode, tests) -----------------------------------------------------
    def _meta(self, tokens: torch.Tensor, positions: list[int], seq: int) -> RowMeta:
        dev = self.device
        m = len(positions)
        return RowMeta(tokens=tokens, token_stride=1,
                       pos=torch.tensor(positions, dtype=torch.int32, device=dev),
                       seq=torch.zeros((m,), dtype=torch.int32, device=dev),
                       seq_rows=torch.tensor([0, m], dtype=torch.int32, device=dev),
                       rows=m, max_rows_per_seq=m,
                       seq_slot=torch.tensor([seq], dtype=torch.int32, device=dev))

    def prefill(self, tokens: torch.Tensor, seq: int = 0, start: int = 0) -> None:
        """Write the KV of `tokens` (int32 on the device) at slots start.. of sequence slot `seq`."""
        total = tokens.numel()
        step = min(self.max_rows, PREFILL_SEQ_ROWS)
        for off in range(0, total, step):
            part = tokens[off:off + step].contiguous()
            meta = self._meta(part, list(range(start + off, start + off + part.numel())), seq)
            self.forward(meta, max_kv_len=self.max_ctx)

    def prefill_many(self, prompts: list[tuple[int, torch.Tensor]]) -> None:
        """Prefill several sequence slots together: each forward packs the next (up to 256-token) chunk of as many
        sequences as fit in max_rows (up to 320 rows), so the projections run at many rows at once. A sequence's
        chunks are the ones `prefill` would cut, and every kernel is row-invariant, so the KV written is the same
        bits as prefilling the sequences one by one. `prompts`: (slot, int32 tokens on the device[, start]), the
        tokens going to slots start.. of the slot (0 by default: the K/V of slots below start are already there)."""
        dev = self.device
        starts = [p[2] if len(p) > 2 else 0 for p in prompts]
        plan = prefill_plan([p[1].numel() for p in prompts], min(self.max_rows, PREFILL_SEQ_ROWS),
                            min(self.max_rows, MAX_QGEMM_ROWS))
        for forward in plan:
            parts = [prompts[i][1][off:off + n] for i, off, n in forward]
            rows = [0]
            for _, _, n in forward:
                rows.append(rows[-1] + n)
            meta = RowMeta(tokens=torch.cat(parts).to(torch.int32).contiguous(), token_stride=1,
                           pos=torch.tensor([starts[i] + p for i, off, n in forward for p in range(off, off + n)],
                                            dtype=torch.int32, device=dev),
                           seq=torch.tensor([g for g, (_, _, n) in enumerate(forward) for _ in range(n)],
                                            dtype=torch.int32, device=dev),
                           seq_rows=torch.tensor(rows, dtype=torch.int32, device=dev), rows=rows[-1],
                           max_rows_per_seq=max(n for _, _, n in forward),
                           seq_slot=torch.tensor([prompts[i][0] for i, _, _ in forward], dtype=torch.int32,
                                                 device=dev))
            self.forward(meta, max_kv_len=self.max_ctx)

    def logits_for(self, tokens: torch.Tensor, start: int, seq: int = 0) -> torch.Tensor:
        """Feed `tokens` (one forward, rows at slots start..) and return every row's logits [M, V]."""
        m = tokens.numel()
        meta = self._meta(tokens.contiguous(), list(range(start, start + m)), seq)
        return self.forward(meta, max_kv_len=self.max_ctx, logit_rows=m)


def prefill_plan(lengths: list[int], step: int, budget: int) -> list[list[tuple[int, int, int]]]:
    """The forwards of a packed prefill: each a list of (prompt index, offset, count). Every prompt advances by
    chunks of `step` tokens (the chunks a one-by-one prefill cuts); a forward takes, in prompt order, the next
    chunk of each unfinished prompt while the rows stay within `budget`."""
    if step < 1 or budget < step:
        raise ValueError("need 1 <= step <= budget")
    offs = [0] * len(lengths)
    plan = []
    while True:
        forward, rows = [], 0
        for i, n in enumerate(lengths):
            if offs[i] >= n:
                continue
            c = min(step, n - offs[i])
            if rows + c > budget:
                break
            forward.append((i, offs[i], c))
            offs[i] += c
            rows += c
        if not forward:
            return plan
        plan.append(forward)


@dataclass
class SpecStats:
    rounds: int = 0
    tokens: int = 0
    accepted: int = 0


@dataclass(frozen=True)
class Sampling:
    """Stochastic speculative decoding: temperature, top-p, and the Philox seed of the whole run."""
    temperature: float = 0.7
    top_p: float = 0.95
    seed: int = 0


DRAFT_DRAW = 1000  # Philox draw of draft pass i is DRAFT_DRAW + i; acceptance uses draws 0 .. 2k


class SpecDecoder:
    """Speculative decoding of `batch` sequences with `k` drafts per round, the round on the device.

    Each sequence slot b holds its committed tokens on the device. A round is: prepare the row buffers; draft
    pass 0 (the last two committed tokens) and passes 1..k-1 (one draft each) through the draft model, each
    followed by a device pick that writes the next draft straight into the verify rows; one verify forward of
    the target over k+1 rows per sequence; acceptance on the device; commit. `capture()` records one round as a
    CUDA graph; `run_rounds(n)` replays it n times with no host synchronisation.

    Greedy (sampling=None): the picks are argmaxes and acceptance keeps the drafts equal to the target's argmax
    (the reference's rule, ironmule/speculation.py:103-108). Stochastic (sampling=Sampling(...)): draft i of
    sequence b is sampled from the draft's temperature/top-p distribution with Philox (seed, offset = round,
    stream = b, draw = DRAFT_DRAW + i), the draft distributions are kept, and acceptance is the p/q rejection
    rule with residual resampling on draws 0 .. 2k of the same stream -- so a round is reproducible from
    (seed, round) and its decisions can be replayed on the CPU. The reference has no stochastic path (its
    product refuses sampling, ironmule_product/worker.py:485-486).
    """

    def __init__(self, target: QuantModel, draft: QuantModel, *, k: int = 4, batch: int = 1,
                 sampling: Sampling | None = None, prefix_cache: bool = False):
        if target.cfg.vocab != draft.cfg.vocab:
            raise ValueError("draft and target must share a vocabulary")
        if batch > min(target.max_seqs, draft.max_seqs):
            raise ValueError("batch exceeds the models' sequence slots")
        if batch * (k + 1) > min(target.max_rows, MAX_QGEMM_ROWS) or batch * (k + 1) > target.max_logit_rows:
            raise ValueError("batch * (k + 1) verify rows exceed the target's per-forward limit")
        if 2 * batch > draft.max_rows or 2 * batch > draft.max_logit_rows:
            raise ValueError("draft pass rows exceed the draft model's limit")
        self.target, self.draft, self.k, self.batch = target, draft, k, batch
        self.reserve = k  # cache slots a round may write past the committed tokens
        dev = target.device
        self.device = dev
        b = batch
        i32 = dict(dtype=torch.int32, device=dev)
        self.cap = min(target.max_ctx, draft.max_ctx)
        self.hist = torch.zeros((b, self.cap), **i32)
        self.n = torch.full((b,), 2, **i32)
        self.target_len = torch.zeros((b,), **i32)
        self.stats = torch.zeros((b, 3), dtype=torch.int64, device=dev)
        self.d0_tok = torch.zeros((2 * b,), **i32)
        self.d0_pos = torch.zeros((2 * b,), **i32)
        self.d_pos = torch.zeros((max(k - 1, 1), b), **i32)
        self.v_tok = torch.zeros((b * (k + 1),), **i32)
        self.v_pos = torch.zeros((b * (k + 1),), **i32)
        self.out_tokens = torch.zeros((b, k + 1), **i32)
        self.out_count = torch.zeros((b,), **i32)
        ar = torch.arange(b, **i32)
        self.seq_d0 = ar.repeat_interleave(2)
        self.rows_d0 = torch.arange(0, 2 * b + 1, 2, **i32)
        self.seq_d = ar.clone()
        self.rows_d = torch.arange(0, b + 1, **i32)
        self.seq_v = ar.repeat_interleave(k + 1)
        self.rows_v = torch.arange(0, b * (k + 1) + 1, k + 1, **i32)
        self.ws_verify = kernels.workspace(kernels.argmax_workspace_bytes(b * (k + 1), target.cfg.vocab), dev)
        self.sampling = sampling
        if sampling is not None:
            v = target.cfg.vocab
            self.dlog = torch.zeros((k, b, v), dtype=torch.bfloat16, device=dev)  # draft pass i's logits per sequence
            self.offset = torch.zeros((1,), dtype=torch.int64, device=dev)         # rounds so far (the Philox offset)
            self.streams = torch.arange(b, dtype=torch.int32, device=dev)
            self.ws_draw = kernels.workspace(kernels.sampling_workspace_bytes(b), dev)
            self.ws_accept = kernels.workspace(kernels.sampling_workspace_bytes(b * (2 * k + 1)), dev)
        self.graph: torch.cuda.CUDAGraph | None = None
        self.gpu_launches_per_round = 0
        self.pool: PagePool | None = None
        if prefix_cache:
            # one page pool over both models' caches (a slot's row lists the same physical pages in each), less
            # PARK_PAGES private pages per slot at the top, where an idle slot's rounds write
            pages = min(target.max_seqs * target.pages_per_seq, draft.max_seqs * draft.pages_per_seq)
            self.park_base = pages - PARK_PAGES * batch
            if self.park_base < 1:
                raise ValueError("the caches are too small for a page pool")
            self.pool = PagePool(self.park_base, batch, min(target.pages_per_seq, draft.pages_per_seq), lead=2)
        # host view of the slots: running or idle (parked), the committed tokens reported so far, the end
        self.running = [False] * batch
        self.upto = [0] * batch
        self.end = [0] * batch
        self.reused = [0] * batch
        self.prefill_tokens = 0
        self._host_n = self._host_tok = None
        for b in range(batch):
            self._park(b)

    # ---- one round, issued on the current stream --------------------------------------------------------
    def round(self) -> None:
        t, d, k, b = self.target, self.draft, self.k, self.batch
        slot_cap = self.cap
        kernels.spec_prepare(self.hist, self.n, self.target_len, b, k, slot_cap, self.d0_tok, self.d0_pos,
                             self.d_pos if k > 1 else None, self.v_tok, self.v_pos)
        # draft pass 0: two rows per sequence; the argmax reads the second row of each pair (the head runs over
        # both: its cost is the weight stream, not the rows)
        meta = RowMeta(self.d0_tok, 1, self.d0_pos, self.seq_d0, self.rows_d0, 2 * b, 2)
        logits = d.forward(meta, max_kv_len=slot_cap, logit_rows=2 * b)
        self._pick(0, logits[1:], 2 * d.cfg.vocab)
        for i in range(1, k):
            meta = RowMeta(self.v_tok[i:], k + 1, self.d_pos[i - 1], self.seq_d, self.rows_d, b, 1)
            logits = d.forward(meta, max_kv_len=slot_cap, logit_rows=b)
            self._pick(i, logits, d.cfg.vocab)
        meta = RowMeta(self.v_tok, 1, self.v_pos, self.seq_v, self.rows_v, b * (k + 1), k + 1)
        logits = t.forward(meta, max_kv_len=slot_cap, logit_rows=b * (k + 1))
        if self.sampling is None:
            kernels.verify_greedy(logits, self.v_tok[1:], b=b, k=k, drafts_ld=k + 1, tokens=self.out_tokens,
                                  count=self.out_count, ws=self.ws_verify)
        else:
            sp = self.sampling
            kernels.accept_stochastic(logits, self.dlog, self.v_tok[1:], b=b, k=k, drafts_ld=k + 1,
                                      temperature=sp.temperature, top_p=sp.top_p, seed=sp.seed,
                                      offset_dev=self.offset, tokens=self.out_tokens, count=self.out_count,
                                      ws=self.ws_accept)
            self.offset.add_(1)
        kernels.spec_commit(self.hist, self.n, self.target_len, b, k, self.out_tokens, self.out_count, self.stats)

    def _pick(self, i: int, logits: torch.Tensor, ld: int) -> None:
        """Draft i of every sequence from the draft logits rows (row b at logits[b * ld]) into the verify rows."""
        b, k = self.batch, self.k
        if self.sampling is None:
            kernels.argmax_rows(logits, out=self.v_tok[i + 1:], out_stride=k + 1, ws=self.draft.ws_argmax, rows=b,
                                ld=ld)
            return
        v = self.draft.cfg.vocab
        self.dlog[i].copy_(logits.as_strided((b, v), (ld, 1)))
        sp = self.sampling
        kernels.sample_rows(self.dlog[i], sp.temperature, sp.top_p, sp.seed, offset_dev=self.offset,
                            streams=self.streams, draw=DRAFT_DRAW + i, out=self.v_tok[i + 1:], out_stride=k + 1,
                            rows=b, ws=self.ws_draw)

    def launches_per_round(self) -> int:
        """libimspec kernel launches in one round (counted from the round's structure)."""
        def fwd(model, logits):
            per_layer = 7 if model.cfg.family == "gemma3" else 5
            return 1 + per_layer * model.cfg.layers + (1 if logits else 0)
        pick, accept = (1, 1) if self.sampling is None else (2, 3)  # argmax | row distributions + sample
        return 1 + self.k * (fwd(self.draft, True) + pick) + fwd(self.target, True) + accept + 1

    # ---- state ------------------------------------------------------------------------------------------
    def start(self, prompts: list[torch.Tensor], max_new: int) -> None:
        """Load prompts (int32 device tensors, length >= 2) into the sequence slots and prefill both models
        with all but the last prompt token."""
        if len(prompts) != self.batch:
            raise ValueError("one prompt per sequence slot")
        for p in prompts:
            self._check_prompt(p.numel(), max_new)
        self.finish()  # the previous requests end (with a page pool their K/V stay cached)
        self._admit([(b, p, max_new) for b, p in enumerate(prompts)])
        self.stats.zero_()
        if self.sampling is not None:
            self.offset.zero_()

    def request_limit(self) -> int:
        """The most prompt + answer tokens one request may have: the cache less the slots a round writes ahead. With
        a page pool a request also takes at most the pool's pages / slots, so every slot's request fits at once
        (sharing only lowers a request's need, and cached pages are evicted on demand)."""
        limit = self.cap - self.reserve - 1
        if self.pool is not None:
            limit = min(limit, self.pool.pages // self.batch * PAGE - self.reserve - 1)
        return limit

    def _check_prompt(self, length: int, max_new: int) -> None:
        if length < 2 or max_new < 1 or length + max_new > self.request_limit():
            raise ValueError("prompt too short or too long for the cache")

    def start_slots(self, items: list[tuple[int, torch.Tensor, int]]) -> None:
        """Start requests (slot, int32 prompt tensor on the device, max_new) in idle slots while the other slots
        keep running: the continuous batching of the reference's step loop (ironmule/ggml_engine.py:1066-1160).
        Between rounds only; a captured graph stays valid (the slot state lives in the same buffers)."""
        seen = set()
        for b, p, max_new in items:
            if not 0 <= b < self.batch or self.running[b] or b in seen:
                raise ValueError(f"slot {b} is not an idle slot")
            seen.add(b)
            self._check_prompt(p.numel(), max_new)
        self._admit(items)

    def stop_slot(self, b: int, keep: bool = True) -> None:
        """End slot b's request between rounds. With a page pool its K/V stay cached (keep) and its pages go back
        to the pool; the idle slot's rounds then write only its private parking pages."""
        if not self.running[b]:
            return
        if self.pool is not None:
            self._retire(b, keep)
        self.running[b] = False
        self._park(b)

    def _park(self, b: int) -> None:
        """An idle slot: two committed tokens and nothing to commit, so its rounds write positions 0 .. PARK_PAGES *
        PAGE - 1 only (at most 2 + 31 tree nodes), which with a page pool map to the slot's own parking pages."""
        self.hist[b, :2] = 0
        self.n[b] = 2
        self.target_len[b] = 2
        if self.pool is not None:
            park = [self.park_base + PARK_PAGES * b + i for i in range(PARK_PAGES)]
            for model in (self.target, self.draft):
                row = park + [park[-1]] * (model.pages_per_seq - PARK_PAGES)
                model.page_table[b].copy_(torch.tensor(row, dtype=torch.int32))

    def _admit(self, items: list[tuple[int, torch.Tensor, int]]) -> None:
        for b, p, max_new in items:
            length = p.numel()
            self.hist[b, :length] = p.to(torch.int32)
            self.n[b] = length
            self.target_len[b] = length + max_new
            self.running[b] = True
            self.upto[b] = length
            self.end[b] = length + max_new
            self.reused[b] = 0
        if self.pool is None:
            body = [(b, p[:-1].to(torch.int32)) for b, p, _ in items]
            self.target.prefill_many(body)
            self.draft.prefill_many(body)
            self.prefill_tokens = sum(p.numel() - 1 for _, p, _ in items)
        else:
            self._start_shared(items)

    def _start_shared(self, items: list[tuple[int, torch.Tensor, int]]) -> None:
        """Admission over the page pool: every slot's pages come from the pool, a prompt's longest full-page prefix
        that an earlier request left in the caches (or that an earlier prompt of this batch writes) is linked into
        its page-table rows instead of computed, and only the rest is prefilled (the reference's prompt-prefix
        sharing, ironmule/ggml_engine.py:352-389 with :870-919). Prompts are prefilled in waves: a prompt that
        would share more pages with an earlier prompt of the batch than the cache offers waits for the wave after
        that prompt's, so every shared page is written before it is read. A slot's K/V are final, and its pages
        are indexed, for the committed tokens but the last two (the first draft pass rewrites the K/V of the
        second-to-last one)."""
        pool = self.pool
        prompts = {b: p for b, p, _ in items}
        ids = {b: p.tolist() for b, p, _ in items}
        limits = {b: max_new + self.reserve + 1 for b, _, max_new in items}

        def common(a: list[int], b: list[int]) -> int:
            n = min(len(a), len(b))
            i = 0
            while i < n and a[i] == b[i]:
                i += 1
            return i

        waiting = [b for b, _, _ in items]
        self.prefill_tokens = 0
        while waiting:
            wave, later = [], []
            for b in waiting:
                room = (len(ids[b]) - pool.lead) // PAGE
                cached = min(len(pool.longest(ids[b])), room)
                mine = max((min(common(ids[b], ids[a]), len(ids[a]) - 2) // PAGE for a in wave), default=0)
                (later if min(mine, room) > cached else wave).append(b)
            body = []
            for b in wave:
                placed = pool.place(ids[b], limits[b], slot=b)
                if placed is None:
                    raise RuntimeError("the page pool cannot hold the batch")
                _, keep = placed
                self.reused[b] = keep
                for model in (self.target, self.draft):
                    row = pool.row(b, model.pages_per_seq)
                    model.page_table[b].copy_(torch.tensor(row, dtype=torch.int32))
                body.append((b, prompts[b][keep:-1].to(torch.int32), keep))
                self.prefill_tokens += len(ids[b]) - 1 - keep
            self.target.prefill_many(body)
            self.draft.prefill_many(body)
            for b in wave:
                pool.commit(b, ids[b][:-2])
            waiting = later

    def _retire(self, b: int, keep: bool = True) -> None:
        """Release slot b's pages to the pool, first indexing those that hold final K/V."""
        n = int(self.n[b].item())
        if keep and n > 2:
            self.pool.commit(b, self.hist[b, :n - 2].tolist())
        self.pool.release(b, keep=keep)

    def finish(self, keep: bool = True) -> None:
        """End every running slot's request (`stop_slot`): with a page pool the K/V of their committed tokens stay
        cached for later requests (keep) or are dropped. `start` does this itself."""
        for b in range(self.batch):
            self.stop_slot(b, keep)

    def step(self) -> dict[int, list[int]]:
        """One round (the captured graph when there is one), then each running slot's newly committed tokens, read
        back to the host with one synchronisation; a slot's tokens stop at its end (prompt + max_new)."""
        if self._host_n is None:
            self._host_n = torch.zeros(self.batch, dtype=torch.int32).pin_memory()
            self._host_tok = torch.zeros((self.batch, self.k + 1), dtype=torch.int32).pin_memory()
        self.run_rounds(1)
        self._host_n.copy_(self.n, non_blocking=True)
        self._host_tok.copy_(self.out_tokens, non_blocking=True)
        torch.cuda.current_stream(self.device).synchronize()
        out = {}
        for b in range(self.batch):
            if not self.running[b]:
                continue
            n_b = min(int(self._host_n[b]), self.end[b])
            new = n_b - self.upto[b]
            if new > 0:
                out[b] = self._host_tok[b, :new].tolist()
                self.upto[b] = n_b
        return out

    def capture(self) -> None:
        """Record one round as a CUDA graph (after one eager round has loaded every kernel)."""
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph):
            self.round()

    def run_rounds(self, rounds: int) -> None:
        for _ in range(rounds):
            if self.graph is not None:
                self.graph.replay()
            else:
                self.round()

    def generate(self, prompts, max_new: int, on_token=None) -> list[list[int]]:
        """The public streaming call: host prompts (lists of token ids, one per sequence slot) in, the generated
        tokens out. Every round's accepted tokens are read back to the host and passed to
        `on_token(seq, tokens)` (the reference's `generate(prompt_ids, max_tokens, on_token)`,
        ironmule_product/ggml_bridge.py:231-270). The round runs as the captured graph when `capture()` was
        called, else eagerly."""
        pinned = [torch.as_tensor(p, dtype=torch.int32).pin_memory() for p in prompts]
        self.start([p.to(self.device, non_blocking=True) for p in pinned], max_new)
        out: list[list[int]] = [[] for _ in range(self.batch)]
        while True:
            for b, toks in self.step().items():
                out[b].extend(toks)
                if on_token is not None:
                    on_token(b, toks)
            if all(self.upto[b] >= self.end[b] for b in range(self.batch)):
                return out

    def done(self) -> bool:
        return bool(torch.all(self.n >= self.target_len).item())

    def read_stats(self) -> SpecStats:
        s = self.stats.sum(dim=0).tolist()
        return SpecStats(rounds=int(s[0]), tokens=int(s[1]), accepted=int(s[2]))

    def generated(self, b: int, prompt_len: int) -> list[int]:
        n = int(self.n[b].item())
        end = min(n, int(self.target_len[b].item()))
        return self.hist[b, prompt_len:end].tolist()


class TreeDecoder(SpecDecoder):
    """Greedy tree speculation of `batch` sequences, the round on the device.

    The draft tree has a static shape: `branch[L]` children per node at depth L + 1 (default 4 x 2 x 2: 4 + 8 +
    16 = 28 nodes). A round: prepare the rows (im_tree_prepare); draft pass 0 re-feeds the last two committed
    tokens of every sequence and its top-branch[0] tokens become depth-1 nodes; each further draft pass runs one
    level's nodes of every sequence (tree-masked attention: a node sees its sequence's committed prefix and its
    own ancestors) and its rows' top-k become the next level; one verify forward of the target over every
    sequence's root and nodes (1 + 28 = 29 rows per sequence); the target's argmax per row and the walk down each
    tree (im_tree_accept) keep the longest agreeing path plus the target's own token; the accepted nodes' K/V move
    to the committed slots in both models (im_tree_compact); commit. A level's rows are gathered from the
    per-sequence tree rows and the top-k children scattered back with fixed index maps. Every kernel is
    row-invariant and a node sees exactly its path, so the tokens equal plain greedy decoding's. BASELINE's
    "16-node ... M=16" cannot describe a 4 x 2 x 2 tree; this build verifies the whole tree (29 rows per sequence).
    """

    def __init__(self, target: QuantModel, draft: QuantModel, *, branch: tuple[int, ...] = (4, 2, 2),
                 batch: int = 1, prefix_cache: bool = False):
        levels = len(branch)
        counts = [math.prod(branch[:i + 1]) for i in range(levels)]
        nodes = sum(counts)
        rows = 1 + nodes
        if rows > MAX_SEQ_ROWS:
            raise ValueError(f"a {rows}-row tree exceeds the {MAX_SEQ_ROWS} rows of one sequence per forward")
        if batch * rows > min(target.max_rows, MAX_QGEMM_ROWS, target.max_logit_rows):
            raise ValueError(f"{batch} trees of {rows} rows exceed the target's per-forward limit")
        if batch * max(counts[:-1] + [2]) > min(draft.max_rows, draft.max_logit_rows):
            raise ValueError("a tree level exceeds the draft model's per-forward limit")
        super().__init__(target, draft, k=levels, batch=batch, prefix_cache=prefix_cache)
        self.branch, self.counts, self.nodes, self.rows = tuple(branch), counts, nodes, rows
        self.first = [sum(counts[:i]) for i in range(levels)]
        self.reserve = nodes
        dev, i32 = self.device, dict(dtype=torch.int32, device=self.device)
        b = batch
        self.t_tok = torch.zeros((b * rows,), **i32)
        self.t_pos = torch.zeros((b * rows,), **i32)
        self.t_slot = torch.zeros((b * rows,), **i32)
        self.t_mask = torch.zeros((b * rows,), dtype=torch.int64, device=dev)
        self.t_base = torch.zeros((b,), **i32)
        self.t_argmax = torch.zeros((b * rows,), **i32)
        self.acc_node = torch.zeros((b * levels,), **i32)
        self.seq_t = torch.arange(b, **i32).repeat_interleave(rows)
        self.rows_t = torch.arange(0, b * rows + 1, rows, **i32)
        ar = torch.arange(b, dtype=torch.int64, device=dev)
        # children of level-L parents (L = -1: the roots) -> their tree rows, parent-major
        self.child_idx = []
        for lv in range(levels):
            parents = 1 if lv == 0 else counts[lv - 1]
            i = torch.arange(parents * branch[lv], dtype=torch.int64, device=dev)
            self.child_idx.append((ar[:, None] * rows + 1 + self.first[lv] + i[None, :]).reshape(-1))
        # the draft pass over level lv - 1's nodes: gather maps, per-level row buffers and sequence groups
        self.level = []
        for lv in range(1, levels):
            cnt = counts[lv - 1]
            idx = (ar[:, None] * rows + 1 + self.first[lv - 1] + torch.arange(cnt, device=dev)[None, :]).reshape(-1)
            bufs = dict(tok=torch.zeros((b * cnt,), **i32), pos=torch.zeros((b * cnt,), **i32),
                        slot=torch.zeros((b * cnt,), **i32),
                        mask=torch.zeros((b * cnt,), dtype=torch.int64, device=dev),
                        seq=torch.arange(b, **i32).repeat_interleave(cnt),
                        seq_rows=torch.arange(0, b * cnt + 1, cnt, **i32), idx=idx, cnt=cnt)
            self.level.append(bufs)
        self.children = torch.zeros((b * max(counts) + b * branch[0],), **i32)
        self.ws_topk = kernels.workspace(
            kernels.topk_workspace_bytes(b * max(counts + [1]), target.cfg.vocab, max(branch)), dev)

    def round(self) -> None:
        t, d, br, b = self.target, self.draft, self.branch, self.batch
        cap, v = self.cap, d.cfg.vocab
        kernels.tree_prepare(self.hist, self.n, br, cap, self.d0_tok, self.d0_pos, self.t_tok, self.t_pos, self.t_slot,
                             self.t_mask, self.t_base)
        meta = RowMeta(self.d0_tok, 1, self.d0_pos, self.seq_d0, self.rows_d0, 2 * b, 2)
        logits = d.forward(meta, max_kv_len=cap, logit_rows=2 * b)
        kids = self.children[:b * br[0]]
        kernels.topk_rows(logits[1:], br[0], rows=b, ld=2 * v, out=kids, ws=self.ws_topk)
        self.t_tok.index_copy_(0, self.child_idx[0], kids)
        for lv in range(1, len(br)):
            L = self.level[lv - 1]
            for key, src in (("tok", self.t_tok), ("pos", self.t_pos), ("slot", self.t_slot), ("mask", self.t_mask)):
                torch.index_select(src, 0, L["idx"], out=L[key])
            n = b * L["cnt"]
            meta = RowMeta(L["tok"], 1, L["pos"], L["seq"], L["seq_rows"], n, L["cnt"], slot=L["slot"],
                           tree_mask=L["mask"], tree_base=self.t_base)
            logits = d.forward(meta, max_kv_len=cap, logit_rows=n)
            kids = self.children[:n * br[lv]]
            kernels.topk_rows(logits, br[lv], rows=n, out=kids, ws=self.ws_topk)
            self.t_tok.index_copy_(0, self.child_idx[lv], kids)
        meta = RowMeta(self.t_tok, 1, self.t_pos, self.seq_t, self.rows_t, b * self.rows, self.rows, slot=self.t_slot,
                       tree_mask=self.t_mask, tree_base=self.t_base)
        logits = t.forward(meta, max_kv_len=cap, logit_rows=b * self.rows)
        kernels.argmax_rows(logits, out=self.t_argmax, ws=t.ws_argmax, rows=b * self.rows)
        kernels.tree_accept(self.t_argmax, self.t_tok, b, br, self.out_tokens, self.out_count, self.acc_node)
        kernels.tree_compact(t.k_cache, t.v_cache, t.page_table, self.t_base, self.acc_node, len(br), len(br), b)
        kernels.tree_compact(d.k_cache, d.v_cache, d.page_table, self.t_base, self.acc_node, len(br), len(br) - 1, b)
        kernels.spec_commit(self.hist, self.n, self.target_len, b, len(br), self.out_tokens, self.out_count,
                            self.stats)

    def launches_per_round(self) -> int:
        def fwd(model):
            return 2 + (7 if model.cfg.family == "gemma3" else 5) * model.cfg.layers
        levels = len(self.branch)
        return 1 + levels * (fwd(self.draft) + 1) + fwd(self.target) + 1 + 1 + 2 + 1


def greedy_decode(model: QuantModel, prompt: torch.Tensor, max_new: int, seq: int = 0) -> list[int]:
    """Plain greedy decoding, one token per forward (the reference's non-speculative step); the baseline
    that speculation must reproduce token for token."""
    prompt = prompt.to(torch.int32)
    model.prefill(prompt[:-1], seq=seq)
    out: list[int] = []
    last = prompt[-1:].clone()
    pos = prompt.numel() - 1
    for _ in range(max_new):
        logits = model.logits_for(last, pos, seq=seq)
        idx, _ = kernels.argmax_rows(logits, ws=model.ws_argmax)
        last = idx.clone()
        out.append(int(idx.item()))
        pos += 1
    return out


# ---- the draft-model protocol of the reference's host speculation, on the device ------------------------------
def decode_plan(wants: list[list[bool]], step: int, budget: int, logit_budget: int
                ) -> list[tuple[list[tuple[int, int, int]], int]]:
    """The forwards of one multi-sequence decode call: `wants[i]` says, per row of sequence i (rows in position
    order), whether it needs logits. Each forward takes at most one chunk of up to `step` rows of each sequence
    (a sequence's chunks in order), at most `budget` rows in all; the chunks that need logits come first so that the
    logits cover a leading block of at most `logit_budget` rows. Returns [(chunks [(sequence, offset, count)],
    logit rows)]."""
    if step < 1 or budget < step or logit_budget < step:
        raise ValueError("need 1 <= step <= budget and step <= logit_budget")
    offs = [0] * len(wants)
    plan = []
    while True:
        ready = []
        for i, w in enumerate(wants):
            if offs[i] < len(w):
                n = min(step, len(w) - offs[i])
                last = max((j for j in range(n) if w[offs[i] + j]), default=-1)
                ready.append((i, offs[i], n, last))
        if not ready:
            return plan
        chunks, rows, logit_rows = [], 0, 0
        for i, off, n, last in [c for c in ready if c[3] >= 0] + [c for c in ready if c[3] < 0]:
            if rows + n > budget or (last >= 0 and rows + last + 1 > logit_budget):
                continue
            if last >= 0:
                logit_rows = rows + last + 1
            chunks.append((i, off, n))
            rows += n
            offs[i] += n
        plan.append((chunks, logit_rows))


class DeviceDraftEngine:
    """A draft model on the B200 behind the engine protocol the reference's `Drafter` drives
    (ironmule/draft_model.py:159-288): `_decode_conf(rows)` takes llama.cpp-style rows (token, position, sequence,
    wants logits) and returns, per row that wants logits, its top token and that token's probability (the
    reference's host scan, ironmule/ggml_engine.py:669-683, here `kernels.argmax_rows(with_conf=True)`); `eog`,
    `L.llama_memory_seq_rm(memory, seq, p0, p1)`, `memory` and `seqs` as the reference's engine has them.

    The cache is indexed by position and a row reads only keys at or below its own position, so removing a
    sequence's tail is bookkeeping: the next rows overwrite those slots. A removal that would leave a hole below
    kept positions answers False, as llama.cpp does for removals its cache cannot make (the `Drafter` then
    clears the sequence). Rows must continue each sequence from its first free position.
    """

    def __init__(self, model: QuantModel, eog_ids=()):
        step = min(model.max_rows, MAX_SEQ_ROWS)
        if model.max_logit_rows < step:
            raise ValueError(f"the draft model needs max_logit_rows >= {step}")
        self.model = model
        self.seqs = model.max_seqs
        self.seq_ctx = model.max_ctx  # positions per sequence (the reference engine's name)
        self.max_rows = min(model.max_rows, model.max_logit_rows, MAX_QGEMM_ROWS)  # rows of one forward with logits
        self.memory = None
        self.filled = [0] * model.max_seqs  # positions of each sequence whose K/V are written
        self.eog_ids = frozenset(int(t) for t in eog_ids)
        self.L = _SeqRm(self)
        self.forwards = 0

    def eog(self, token: int) -> bool:
        return int(token) in self.eog_ids

    def seq_rm(self, seq: int, p0: int, p1: int) -> bool:
        if not 0 <= seq < self.seqs:
            raise ValueError(f"sequence {seq} out of range")
        start = 0 if p0 < 0 else p0
        if 0 <= p1 < self.filled[seq] and start < p1:
            return False
        self.filled[seq] = min(self.filled[seq], start)
        return True

    def _decode_conf(self, rows) -> list[tuple[int, float]]:
        if not rows:
            return []
        m = self.model
        per: dict[int, list[int]] = {}
        for i, (_, pos, seq, _) in enumerate(rows):
            if not 0 <= seq < self.seqs:
                raise ValueError(f"sequence {seq} out of range")
            per.setdefault(seq, []).append(i)
        seqs = list(per)
        for seq in seqs:
            first = self.filled[seq]
            for j, i in enumerate(per[seq]):
                if rows[i][1] != first + j:
                    raise ValueError(f"sequence {seq}: row at position {rows[i][1]}, expected {first + j}")
            if first + len(per[seq]) > m.max_ctx:
                raise ValueError(f"sequence {seq} would exceed the model's {m.max_ctx} positions")
        plan = decode_plan([[bool(rows[i][3]) for i in per[s]] for s in seqs], min(m.max_rows, MAX_SEQ_ROWS),
                           min(m.max_rows, MAX_QGEMM_ROWS), m.max_logit_rows)
        picks, where = [], {}
        for chunks, logit_rows in plan:
            order = [per[seqs[g]][off + j] for g, off, n in chunks for j in range(n)]
            bounds = [0]
            for _, _, n in chunks:
                bounds.append(bounds[-1] + n)
            host = ([int(rows[i][0]) for i in order] + [int(rows[i][1]) for i in order]
                    + [g for g, (_, _, n) in enumerate(chunks) for _ in range(n)] + bounds
                    + [seqs[g] for g, _, _ in chunks])
            dev = torch.tensor(host, dtype=torch.int32).to(m.device)
            r, c = len(order), len(chunks)
            meta = RowMeta(tokens=dev[:r], token_stride=1, pos=dev[r:2 * r], seq=dev[2 * r:3 * r],
                           seq_rows=dev[3 * r:3 * r + c + 1], rows=r, max_rows_per_seq=max(n for _, _, n in chunks),
                           seq_slot=dev[3 * r + c + 1:])
            logits = m.forward(meta, max_kv_len=m.max_ctx, logit_rows=logit_rows)
            self.forwards += 1
            if logit_rows:
                idx, conf = kernels.argmax_rows(logits, with_conf=True, ws=m.ws_argmax)
                for k, i in enumerate(order[:logit_rows]):
                    if rows[i][3]:
                        where[i] = (len(picks), k)
                picks.append((idx, conf))
            for g, off, n in chunks:
                self.filled[seqs[g]] += n
        if not picks:
            return []
        idx = torch.cat([p[0] for p in picks]).cpu().tolist()
        conf = torch.cat([p[1] for p in picks]).cpu().tolist()
        base = [0]
        for p in picks:
            base.append(base[-1] + p[0].numel())
        out = []
        for i, row in enumerate(rows):
            if row[3]:
                f, k = where[i]
                out.append((int(idx[base[f] + k]), float(conf[base[f] + k])))
        return out


class _SeqRm:
    """The `L` namespace of the engine protocol: llama.cpp's `llama_memory_seq_rm(memory, seq, p0, p1)`."""

    def __init__(self, engine: DeviceDraftEngine):
        self._e = engine

    def llama_memory_seq_rm(self, memory, seq: int, p0: int, p1: int) -> bool:
        return self._e.seq_rm(seq, p0, p1)


def drafter_generate(target: QuantModel, drafter, prompt, max_new: int, *, max_drafts: int = 8, seq: int = 0,
                     key: int = 0) -> tuple[list[int], dict]:
    """Greedy speculative decoding of one request with the reference's host loop around a `Drafter`
    (ironmule_b200.draft_model, over a `DeviceDraftEngine`): each step the drafter offers as many drafts as its
    confidence-calibrated stop rule gives (0 .. max_drafts), the target verifies the last token and the drafts
    in one forward at their positions, the leading drafts equal to the target's argmax are kept with the target's
    own next token (`speculation.accept`), and the drafter learns from the outcome (`settle`, `end_step`) --
    the per-request step of ironmule/ggml_engine.py:1155-1343 with one running request. Returns the generated
    tokens (exactly max_new, equal to plain greedy decoding) and counts."""
    import time

    from .speculation import accept

    prompt = [int(t) for t in prompt]
    if len(prompt) < 2:
        raise ValueError("a prompt of at least two tokens")
    limit = min(target.max_logit_rows, target.max_rows, MAX_SEQ_ROWS) - 1  # the verify forward's rows, minus one
    max_drafts = max(0, min(max_drafts, limit))
    if len(prompt) + max_new + max_drafts + 1 > target.max_ctx:
        raise ValueError("prompt and answer exceed the target's context")
    dev = target.device
    target.prefill(torch.tensor(prompt[:-1], dtype=torch.int32, device=dev), seq=seq)
    context, out = list(prompt), []
    steps = drafted = accepted = 0
    while len(out) < max_new:
        started = time.perf_counter()
        room = min(max_drafts, max_new - len(out) - 1)
        drafts = drafter.draft({key: (context, room)}, running=1).get(key, []) if room > 0 else []
        feed = torch.tensor([context[-1]] + drafts, dtype=torch.int32, device=dev)
        logits = target.logits_for(feed, len(context) - 1, seq=seq)
        argmax, _ = kernels.argmax_rows(logits, ws=target.ws_argmax)
        new = accept(drafts, argmax.cpu().tolist())
        if drafts:
            drafter.settle(key, len(drafts), len(new) - 1)
        drafter.end_step(time.perf_counter() - started, 1, len(drafts), len(new))
        steps, drafted, accepted = steps + 1, drafted + len(drafts), accepted + len(new) - 1
        context += new
        out += new
    drafter.release(key)
    return out[:max_new], {"steps": steps, "drafted": drafted, "accepted": accepted}
