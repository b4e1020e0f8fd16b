"""Batched generate_batch_ids on the paged pool.

The reference's ``LlamaInferenceEngine.generate_batch_ids``
(src/inference.py:415-457) serves a batch by running ``generate_ids`` for one
prompt after another: every token of every sequence is one pass over all layers
(``forward_layer_cached`` per layer, src/layer.py:221-263), then the final
RMSNorm and the LM head on the last position (src/inference.py:233-253) and the
sampler.  ``BatchGenerator`` produces the same tokens with every sequence of the
batch advancing together:

* each prompt is prefilled into its own block-table rows of one paged pool
  (``paged.BatchDecoder.prefill``, chunked like ``prefill_tokens`` when asked);
* then every decode step runs all sequences' next tokens through each layer in
  one ``kvc_forward_layer_paged`` call (``BatchDecoder.step``), the final RMSNorm
  (``kvc_rmsnorm``) and the LM head (``kvc_linear``) on the whole batch, and the
  sampler per sequence.

Greedy decoding (temperature 0, no repetition penalty) takes the argmax of each
sequence's fp16 logits, as ``sample_next_token`` does (src/inference.py:51-121).
Any other sampling goes through a caller-supplied ``sampler`` with that
function's signature (the reference's own ``sample_next_token``), fed each
sequence's logits on the host and a ``numpy`` generator seeded ``seed + i`` for
prompt i, exactly like the sequential loop.  A sequence that has stopped (EOS)
keeps riding along in the batch; its extra tokens are discarded.
"""

from __future__ import annotations

import time
from dataclasses import dataclass
from typing import Callable, Dict, List, Optional, Sequence, Tuple

import numpy as np
import torch

import kvcache_ffi as ffi
import paged

# GGUF names of one layer's projections in forward_layer_cached's order
_PROJ = ["attn_q", "attn_k", "attn_v", "attn_output", "ffn_gate", "ffn_up", "ffn_down"]
# GGML type ids the kernels take (KVC_WTYPE_*); F32 (0) is converted to F16
_F32, _F16 = 0, 1
_KERNEL_TYPES = {1, 2, 8, 12, 14}


@dataclass
class ModelConfig:
    layers: int
    hidden: int
    intermediate: int
    heads: int
    kv_heads: int
    head_dim: int
    vocab: int
    eps: float = 1e-5
    rope_base: float = 10000.0
    rope_neox: bool = False
    eos_token_id: int = -1


def _f16_rows(raw: np.ndarray, typ: int, n: int, k: int) -> np.ndarray:
    if typ == _F16:
        return np.frombuffer(memoryview(np.ascontiguousarray(raw)), dtype=np.float16).reshape(n, k)
    if typ == _F32:
        return np.frombuffer(memoryview(np.ascontiguousarray(raw)), dtype=np.float32).reshape(n, k).astype(np.float16)
    raise ValueError(f"GGML type {typ} is not a float table")


class BatchModel:
    """The weights generation needs, resident on one GPU: per layer the two norm
    weights and the seven GGML-typed projections (paged.DeviceLayerWeights), the
    token-embedding table as fp16 rows, the output norm and the LM head."""

    def __init__(self, cfg: ModelConfig, layers: List[paged.DeviceLayerWeights],
                 embedding: torch.Tensor, out_norm: torch.Tensor, head: torch.Tensor,
                 head_type: int, device: int):
        self.cfg, self.layers, self.embedding = cfg, layers, embedding
        self.out_norm, self.head, self.head_type, self.device = out_norm, head, head_type, device

    @classmethod
    def from_tensors(cls, cfg: ModelConfig, tensors: Dict[str, Tuple[np.ndarray, int, tuple]],
                     embedding: Optional[np.ndarray] = None, device: int = 0) -> "BatchModel":
        """tensors: GGUF name -> (raw bytes, GGML type id, (n, k) row-major shape),
        the layout of a llama GGUF file (``token_embd.weight``, ``blk.{l}.*``,
        ``output_norm.weight``, ``output.weight``, or the tied embedding).  The
        embedding table is given as fp16 rows when ``token_embd.weight`` is
        quantized (the reference dequantizes rows with its own code)."""
        dev = torch.device("cuda", device)

        def to_dev(a: np.ndarray) -> torch.Tensor:
            return torch.from_numpy(np.ascontiguousarray(a)).to(dev)

        def weight(name: str):
            raw, typ, shape = tensors[name]
            n, k = shape
            if typ == _F32:
                raw, typ = _f16_rows(raw, typ, n, k).view(np.uint8).reshape(-1), _F16
            if typ not in _KERNEL_TYPES:
                raise ValueError(f"{name}: GGML type {typ} is not supported by the kernels")
            return to_dev(np.frombuffer(memoryview(np.ascontiguousarray(raw)), dtype=np.uint8)), typ

        def norm(name: str) -> torch.Tensor:
            raw, typ, shape = tensors[name]
            return to_dev(_f16_rows(raw, typ, 1, cfg.hidden).reshape(-1))

        layers = []
        for l in range(cfg.layers):
            p = f"blk.{l}."
            ws = [weight(p + n + ".weight") for n in _PROJ]
            layers.append(paged.DeviceLayerWeights(norm(p + "attn_norm.weight"),
                                                   norm(p + "ffn_norm.weight"),
                                                   [w for w, _ in ws], [t for _, t in ws],
                                                   cfg.hidden, cfg.intermediate))
        if embedding is None:
            raw, typ, shape = tensors["token_embd.weight"]
            embedding = _f16_rows(raw, typ, shape[0], shape[1])
        if embedding.shape != (cfg.vocab, cfg.hidden):
            raise ValueError(f"the embedding table is {embedding.shape}, expected "
                             f"({cfg.vocab}, {cfg.hidden})")
        head_name = "output.weight" if "output.weight" in tensors else "token_embd.weight"
        head, head_type = weight(head_name)
        if cfg.vocab % 16:
            raise ValueError("the LM head kernel needs a vocabulary that is a multiple of 16")
        return cls(cfg, layers, to_dev(np.asarray(embedding, np.float16)),
                   norm("output_norm.weight"), head, head_type, device)

    @classmethod
    def from_reference_engine(cls, engine, device: int = 0) -> "BatchModel":
        """The weights of a gfx1150-inference ``LlamaInferenceEngine`` moved to the
        GPU once (see ``tensors_from_reference_engine``)."""
        cfg, tensors, embedding = tensors_from_reference_engine(engine)
        return cls.from_tensors(cfg, tensors, embedding=embedding, device=device)


def tensors_from_reference_engine(engine):
    """(ModelConfig, tensors, embedding rows) of a gfx1150-inference
    ``LlamaInferenceEngine``: its layer configuration (LlamaLayerConfig), every
    tensor of its GGUF file read through its WeightStreamer, and the token
    embedding dequantized row by row with the engine's own ``embed_tokens``
    (src/tokenizer.py:336).  Host memory only."""
    import sys

    lc = engine.layer_cfg
    gg = engine.streamer.gguf
    tensors = {}
    for name, info in gg.tensors.items():
        view = np.array(engine.streamer.get_tensor_view(name), copy=True)
        shape = tuple(int(d) for d in info.shape_row_major)
        tensors[name] = (view.view(np.uint8).reshape(-1), int(info.ggml_type), shape)
    mod = sys.modules[type(engine).__module__]
    emb_info = gg.tensors["token_embd.weight"]
    vocab = int(emb_info.shape_row_major[0])
    embedding = mod.embed_tokens(list(range(vocab)), emb_info,
                                 engine.streamer.get_tensor_view("token_embd.weight"),
                                 lc.hidden_size)
    tok = getattr(engine, "tokenizer", None)
    cfg = ModelConfig(layers=int(engine.num_layers), hidden=lc.hidden_size,
                      intermediate=lc.intermediate_size, heads=lc.num_heads,
                      kv_heads=lc.num_kv_heads, head_dim=lc.head_dim, vocab=vocab,
                      eps=float(lc.rms_norm_eps), rope_base=float(lc.rope_freq_base),
                      rope_neox=bool(lc.rope_neox),
                      eos_token_id=int(tok.eos_token_id) if tok is not None else -1)
    return cfg, tensors, np.asarray(embedding, np.float16)


class BatchGenerator:
    """generate_batch_ids for a batch of up to ``max_batch`` prompts of up to
    ``max_seq_len`` positions (prompt + new tokens), on one paged pool."""

    def __init__(self, model: BatchModel, max_batch: int, max_seq_len: int, page_size: int = 16):
        cfg = model.cfg
        self.model, self.max_batch, self.max_seq_len = model, int(max_batch), int(max_seq_len)
        self.pages_per_seq = (self.max_seq_len + page_size - 1) // page_size
        self.pool = paged.PagedKVCache(cfg.layers, self.max_batch * self.pages_per_seq, page_size,
                                       cfg.kv_heads, cfg.head_dim, dtype=torch.float16,
                                       device=model.device)
        table = np.arange(self.max_batch * self.pages_per_seq, dtype=np.int32)
        self.bt = torch.from_numpy(table.reshape(self.max_batch, self.pages_per_seq)).to(
            torch.device("cuda", model.device))

    def _logits(self, h: torch.Tensor, stream) -> torch.Tensor:
        """Final RMSNorm and LM head of rows h (m, hidden) -> fp16 logits (m, vocab)."""
        m = self.model
        n = int(h.shape[0])
        normed = torch.empty_like(h)
        sp = int(stream.cuda_stream) or None
        ffi.check(ffi.lib.kvc_rmsnorm(int(h.data_ptr()), None, None, int(m.out_norm.data_ptr()),
                                      int(normed.data_ptr()), n, m.cfg.hidden, float(m.cfg.eps),
                                      sp))
        logits = torch.empty((n, m.cfg.vocab), dtype=torch.float16, device=h.device)
        ffi.check(ffi.lib.kvc_linear(int(normed.data_ptr()), n, m.cfg.hidden,
                                     int(m.head.data_ptr()), m.head_type, m.cfg.vocab,
                                     int(logits.data_ptr()), sp))
        return logits

    def generate_batch_ids(
        self,
        batch_prompt_ids: Sequence[Sequence[int]],
        max_new_tokens: int = 16,
        temperature: float = 0.0,
        top_k: int = 40,
        top_p: float = 0.95,
        repetition_penalty: float = 1.0,
        stop_on_eos: bool = True,
        seed: Optional[int] = 42,
        prefill_chunk_size: Optional[int] = None,
        sampler: Optional[Callable] = None,
    ) -> Tuple[List[List[int]], Dict[str, float]]:
        """The arguments and result of the reference's generate_batch_ids
        (src/inference.py:415-457): the generated ids of each prompt and batch
        metrics.  ``sampler`` (the reference's sample_next_token) is required
        unless decoding is greedy (temperature 0, repetition penalty 1)."""
        cfg = self.model.cfg
        prompts = [[int(t) for t in p] for p in batch_prompt_ids]
        b = len(prompts)
        if b > self.max_batch:
            raise ValueError(f"{b} prompts exceed the generator's max_batch {self.max_batch}")
        if max_new_tokens < 0:
            raise ValueError(f"max_new_tokens must be >= 0 (got {max_new_tokens})")
        for p in prompts:
            if not p:
                raise ValueError("prompt_ids must not be empty")
            if len(p) + max_new_tokens > self.max_seq_len:
                raise ValueError(f"len(prompt_ids) ({len(p)}) + max_new_tokens ({max_new_tokens}) "
                                 f"exceeds max_seq_len ({self.max_seq_len})")
            if min(p) < 0 or max(p) >= cfg.vocab:
                raise ValueError("a token id is outside the vocabulary")
        greedy = (temperature == 0.0 or top_k == 1) and repetition_penalty == 1.0
        if not greedy and sampler is None:
            raise ValueError("non-greedy decoding needs sampler= (e.g. the reference's "
                             "sample_next_token)")
        t0 = time.perf_counter()
        outs: List[List[int]] = [[] for _ in range(b)]
        if b == 0 or max_new_tokens == 0:
            return outs, {"batch_size": float(b), "total_tokens_generated": 0.0,
                          "total_time_s": 0.0, "tokens_per_sec": 0.0}
        stream = torch.cuda.current_stream(self.model.device)
        rngs = [np.random.default_rng(None if seed is None else seed + i) for i in range(b)]
        hist = [list(p) for p in prompts]
        dec = paged.BatchDecoder(self.pool, self.model.layers, self.bt[:b].contiguous(),
                                 cfg.heads, [0] * b, eps=cfg.eps, freq_base=cfg.rope_base,
                                 neox=cfg.rope_neox)
        emb = self.model.embedding

        def pick(logits: torch.Tensor) -> List[int]:
            if greedy:
                return [int(t) for t in torch.argmax(logits.float(), dim=1).tolist()]
            host = logits.cpu().numpy()
            return [int(sampler(host[i], temperature=temperature, top_k=top_k, top_p=top_p,
                                repetition_penalty=repetition_penalty, generated_ids=hist[i],
                                rng=rngs[i])) for i in range(b)]

        try:
            last = []
            for i, p in enumerate(prompts):  # prefill, full or chunked (prefill_tokens)
                ids = torch.tensor(p, dtype=torch.long, device=emb.device)
                step = len(p) if not prefill_chunk_size or prefill_chunk_size <= 0 else prefill_chunk_size
                for s0 in range(0, len(p), step):
                    h = dec.prefill(i, emb[ids[s0:s0 + step]].contiguous(), stream=stream)
                last.append(h[-1:])
            nxt = pick(self._logits(torch.cat(last), stream))
            done = [False] * b
            for i in range(b):
                outs[i].append(nxt[i])
                hist[i].append(nxt[i])
            for _ in range(max_new_tokens - 1):
                for i in range(b):
                    if stop_on_eos and outs[i][-1] == cfg.eos_token_id:
                        done[i] = True
                if all(done):
                    break
                ids = torch.tensor([o[-1] for o in outs], dtype=torch.long, device=emb.device)
                h = dec.step(emb[ids].contiguous(), stream=stream)
                nxt = pick(self._logits(h, stream))
                for i in range(b):
                    if not done[i]:
                        outs[i].append(nxt[i])
                        hist[i].append(nxt[i])
        finally:
            dec.close()
        t = time.perf_counter() - t0
        total = float(sum(len(o) for o in outs))
        return outs, {"batch_size": float(b), "total_tokens_generated": total,
                      "total_time_s": t, "tokens_per_sec": total / max(t, 1e-9)}

    def close(self):
        self.pool.close()
