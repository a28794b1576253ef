"""Rollout engines: the token-level LLM generator and the reference's
string-level ``RolloutEngine``.

:class:`LLMGenerator` runs its own decode loop on the turbol_b200 kernels (no
vLLM): a paged KV cache (16-token blocks, block tables from the native
``KVBlockManager``), prompt-prefix sharing (the G samples of a prompt point
their first block-table entries at the prompt's blocks), prefill through the
flash-attention kernel, and a decode step — embedding, per layer RMSNorm, QKV
GEMM (+bias), RoPE, KV write, paged GQA decode attention, output GEMM
(+residual), RMSNorm, gate/up GEMM with fused SwiGLU, down GEMM (+residual),
final norm, LM-head GEMM, sampling (temperature; top-k, top-p and an
end-of-sequence stop through the filtered sampler) — captured once as a CUDA
graph and replayed per token.  The sampled tokens and their log-probabilities land
in [B, max_new] device matrices (the column comes from a device counter).

:class:`RolloutEngine` keeps the reference's API
(turbol_vllm/include/turbol/rollout/rollout_engine.hpp:8-36:
RolloutConfig{inference_backend, model_path, tensor_parallel_size,
max_new_tokens, temperature, top_p, top_k, max_batch_size}; initialize,
shutdown, generate, generate_batch, is_vllm_available).  Backends: "native"
(LLMGenerator over a byte-level tokenizer; with random weights the text is
noise, the API and throughput are real), "echo" (the reference's fallback,
turbol_vllm/src/rollout/rollout_engine.cpp:42-44) and "vllm" (optional, via
``turbol_b200.vllm_inference``).
"""
from __future__ import annotations

import math
from dataclasses import dataclass
from typing import List, Optional

import torch

from .._native import core as _core, ops as _ops
from ..models.llm import DecoderLM, LMConfig


class LLMGenerator:
    def __init__(self, model: DecoderLM, max_batch: int, max_len: int, block_size: int = 16, seed: int = 0,
                 cuda_graph: bool = True, decode_gemm: Optional[bool] = None, attn_split: int = 1):
        self.m = model
        self.cfg = model.cfg
        self.device = model.device
        self.max_batch, self.max_len, self.bs = max_batch, max_len, block_size
        self.seed = seed
        self.cuda_graph = cuda_graph
        # which layer projections of a decode step run on the weight-stationary
        # decode GEMM (gemm_decode.cu) instead of the general tcgen05 GEMM:
        # None = by batch size as measured on B200 (all four up to 64
        # sequences; beyond that the down projection only, the general GEMM
        # being as fast or faster for QKV, O and gate/up); True / False = all / none
        self.decode_gemm = decode_gemm
        # context chunks per (sequence, KV head) in the decode attention: 1 =
        # one CTA per context (measured fastest: splitting 512 sequences into 3
        # chunks each took the GRPO rollout from 2.21 s to 2.94 s, the chunks'
        # pipeline fill outweighing the fuller last wave); 0 = the wave model of
        # decode_attention_splits; n > 1 = n chunks
        self.attn_split = attn_split
        cfg = self.cfg
        self.blocks_per_seq = (max_len + block_size - 1) // block_size
        # worst case: every sequence private (no sharing) -> max_batch * blocks
        self.num_blocks = max_batch * self.blocks_per_seq + 1
        self.kv = _core().KVBlockManager(self.num_blocks, block_size)
        shape = (self.num_blocks, cfg.n_kv_heads, block_size, cfg.head_dim)
        self.kc = [torch.empty(shape, device=self.device, dtype=torch.bfloat16) for _ in model.layers]
        self.vc = [torch.empty(shape, device=self.device, dtype=torch.bfloat16) for _ in model.layers]
        self._graph = None
        self._graph_B = None
        self.calls = 0

    def reset_graph(self):
        """Drops the captured decode step.  The capture holds the model's weight
        and KV-cache addresses: call this after rebinding the model's storage."""
        self._graph = None
        self._graph_B = None

    # ------------------------------------------------------------ block tables
    def _tables(self, P: int, G: int, Lp: int, steps: int):
        """Block tables with the prompt blocks shared by the G samples of a prompt."""
        self.kv.reset()
        bs = self.bs
        n_prompt_blocks = Lp // bs  # full prompt blocks are shared; a partial one is copied per sample
        tail = Lp - n_prompt_blocks * bs
        B = P * G
        table = torch.zeros(B, self.blocks_per_seq, dtype=torch.int32)
        pre_table = torch.zeros(P, self.blocks_per_seq, dtype=torch.int32)
        for p in range(P):
            st = self.kv.allocate(p, max(Lp, 1))
            if not st.ok():
                raise RuntimeError(f"KV cache: {st}")
            pblocks = self.kv.block_table(p)
            pre_table[p, : len(pblocks)] = torch.tensor(pblocks, dtype=torch.int32)
            for g in range(G):
                s = p * G + g
                sid = P + s
                need = Lp + steps - n_prompt_blocks * bs
                st = self.kv.allocate(sid, max(need, 1))
                if not st.ok():
                    raise RuntimeError(f"KV cache: {st}")
                own = self.kv.block_table(sid)
                row = pblocks[:n_prompt_blocks] + own
                table[s, : len(row)] = torch.tensor(row[: self.blocks_per_seq], dtype=torch.int32)
        return table.to(self.device), pre_table.to(self.device), n_prompt_blocks, tail

    # ------------------------------------------------------------ decode step
    def _decode_step(self, B: int):
        o = _ops()
        cfg, m = self.cfg, self.m
        H, D = cfg.hidden, cfg.head_dim
        st = self.state
        x = st["x"]
        o.embed_fwd(st["tok"], m.s["embed"], x)
        h, qkv, attn, x2, act = st["h"], st["qkv"], st["attn"], st["x2"], st["act"]
        # few sequences: the projections have few output tiles and long K, so
        # split K over the SMs (partials in this workspace); many sequences:
        # the narrow-tile plan without splitting is faster
        ws = st.get("ws")
        kw = {"workspace": ws} if ws is not None else {}
        kw_down = {"workspace": st["ws_down"]} if "ws_down" in st else kw
        scale = 1.0 / math.sqrt(D)
        dg, dg_down = self._decode_gemm_use(B)
        for li, i in enumerate(m.layers):
            P = f"l{i}."
            o.rmsnorm_fwd(x, m.f32[P + "ln1"], h, None, cfg.rms_eps)
            if dg:
                if cfg.qkv_bias:
                    o.gemm_decode(h, m.s[P + "wqkv"], qkv, bias=m.f32[P + "bqkv"], epi=o.EPI_BIAS)
                else:
                    o.gemm_decode(h, m.s[P + "wqkv"], qkv)
            elif cfg.qkv_bias:
                o.gemm(h, m.s[P + "wqkv"], qkv, bias=m.f32[P + "bqkv"], epi=o.EPI_BIAS, **kw)
            else:
                o.gemm(h, m.s[P + "wqkv"], qkv, **kw)
            o.rope_kv_write(qkv, st["pos"], m.table, cfg.n_heads, cfg.n_kv_heads, D, st["seq"], st["table"],
                            self.kc[li], self.vc[li], self.bs)
            o.decode_attention(qkv, self.kc[li], self.vc[li], st["table"], st["ctx"], attn, cfg.n_heads,
                               cfg.n_kv_heads, D, self.bs, scale, st["attn_split"], st.get("attn_part"),
                               st.get("attn_cnt"))
            if dg:
                o.gemm_decode(attn, m.s[P + "wo"], x2, aux=x, epi=o.EPI_RESIDUAL)
                o.rmsnorm_fwd(x2, m.f32[P + "ln2"], h, None, cfg.rms_eps)
                o.gemm_decode(h, m.s[P + "wgu"], act, epi=o.EPI_SWIGLU)
            else:
                o.gemm(attn, m.s[P + "wo"], x2, aux=x, epi=o.EPI_RESIDUAL, **kw)
                o.rmsnorm_fwd(x2, m.f32[P + "ln2"], h, None, cfg.rms_eps)
                o.gemm(h, m.s[P + "wgu"], act, epi=o.EPI_SWIGLU)
            if dg_down:
                o.gemm_decode(act, m.s[P + "wdown"], x, aux=x2, epi=o.EPI_RESIDUAL)
            else:
                o.gemm(act, m.s[P + "wdown"], x, aux=x2, epi=o.EPI_RESIDUAL, **kw_down)
        o.rmsnorm_fwd(x, m.f32["norm"], h, None, cfg.rms_eps)
        o.gemm(h, m.head_weight(), st["logits"])
        self._sample(st)
        st["pos"].add_(1)
        st["ctx"].add_(1)
        o.counter_add(st["step"], 1)

    # ------------------------------------------------------------ sampling
    sampling = (-1, 1.0, -1, 0)  # (top_k, top_p, eos_id, pad_id): plain temperature sampling

    def _filtered(self) -> bool:
        k, p, eos, _ = self.sampling
        return k > 0 or p < 1.0 or eos >= 0

    def _sample(self, st, seed: Optional[int] = None, temperature: Optional[float] = None):
        """Samples st["tok"] from st["logits"] into column st["step"] of the
        generation matrices.  Without explicit seed / temperature they are read
        from device memory (the captured decode step)."""
        o = _ops()
        dev_args = {} if seed is not None else {"seed_t": st["seed_t"], "temp_t": st["temp_t"]}
        t = 1.0 if temperature is None else temperature
        sd = 0 if seed is None else seed
        if self._filtered():
            k, p, eos, pad = self.sampling
            o.sample_filtered(st["logits"], t, k, p, sd, st["step"], 0, st["tok"], None, st["tok_mat"], st["lp_mat"],
                              eos_id=eos, pad_id=pad, done=st["done"], lengths=st["lengths"], n_done=st["n_done"],
                              **dev_args)
        else:
            o.sample(st["logits"], t, sd, st["step"], 0, st["tok"], None, st["tok_mat"], st["lp_mat"], **dev_args)

    def _alloc_state(self, B: int, steps: int):
        cfg = self.cfg
        dev = self.device
        bf = dict(device=dev, dtype=torch.bfloat16)
        return {
            "x": torch.empty(B, cfg.hidden, **bf), "h": torch.empty(B, cfg.hidden, **bf),
            "qkv": torch.empty(B, cfg.qkv_dim, **bf), "attn": torch.empty(B, cfg.q_dim, **bf),
            "x2": torch.empty(B, cfg.hidden, **bf), "act": torch.empty(B, cfg.ffn, **bf),
            "logits": torch.empty(B, cfg.vocab, **bf),
            "tok": torch.zeros(B, device=dev, dtype=torch.int32),
            "pos": torch.zeros(B, device=dev, dtype=torch.int32),
            "ctx": torch.zeros(B, device=dev, dtype=torch.int32),
            "seq": torch.arange(B, device=dev, dtype=torch.int32),
            "table": torch.zeros(B, self.blocks_per_seq, device=dev, dtype=torch.int32),
            "step": torch.zeros(1, device=dev, dtype=torch.int64),
            "tok_mat": torch.zeros(B, steps, device=dev, dtype=torch.int32),
            "lp_mat": torch.zeros(B, steps, device=dev, dtype=torch.float32),
            # sampling seed and temperature live on the device so that one
            # captured decode step serves every generate call
            "seed_t": torch.zeros(1, device=dev, dtype=torch.int64),
            "temp_t": torch.ones(1, device=dev, dtype=torch.float32),
            # end-of-sequence state (used when an eos_id is given)
            "done": torch.zeros(B, device=dev, dtype=torch.uint8),
            "lengths": torch.full((B,), steps, device=dev, dtype=torch.int32),
            "n_done": torch.zeros(1, device=dev, dtype=torch.int32),
            **self._split_workspace(B),
            **self._attn_split_state(B),
        }

    def _attn_split_state(self, B: int) -> dict:
        """Context split of the decode attention (``attn_split``), with the
        merge scratch."""
        cfg, o = self.cfg, _ops()
        G = cfg.n_heads // cfg.n_kv_heads
        want = getattr(self, "attn_split", 1)
        if want == 1 or self.bs != 16 or cfg.head_dim != 128 or G > 8 or cfg.n_heads % cfg.n_kv_heads:
            return {"attn_split": 1}
        n = int(o.decode_attention_splits(B, cfg.n_kv_heads)) if want == 0 else int(want)
        if n <= 1:
            return {"attn_split": 1}
        return {"attn_split": n,
                "attn_part": torch.empty(o.decode_attention_part_numel(B, cfg.n_heads, cfg.n_kv_heads, n),
                                         device=self.device),
                "attn_cnt": torch.zeros(B * cfg.n_kv_heads, device=self.device, dtype=torch.int32)}

    def _decode_gemm_use(self, B: int):
        """(QKV / O / gate-up on the decode GEMM, down projection on it)."""
        if self.decode_gemm is not None:
            return bool(self.decode_gemm), bool(self.decode_gemm)
        return B <= 64, True

    def _split_workspace(self, B: int) -> dict:
        """Split-K partials of the general GEMM, for the projections it runs."""
        o, cfg = _ops(), self.cfg
        dg, dg_down = self._decode_gemm_use(B)
        if (B > 64 and dg_down) or (B <= 64 and dg):
            return {}
        if B > 64:
            # many sequences: only the down projection (long K = ffn, few output
            # tiles) gains from splitting K; the others keep the narrow-tile plan
            return {"ws_down": torch.zeros(max(o.gemm_workspace_numel(B, cfg.hidden, cfg.ffn), 1), device=self.device)}
        n = max(o.gemm_workspace_numel(B, cfg.qkv_dim, cfg.hidden), o.gemm_workspace_numel(B, cfg.hidden, cfg.q_dim),
                o.gemm_workspace_numel(B, cfg.hidden, cfg.ffn), 1)
        return {"ws": torch.zeros(n, device=self.device)}

    # ------------------------------------------------------------ generate
    @torch.no_grad()
    def generate(self, prompts: torch.Tensor, group: int = 1, max_new: int = 16, temperature: float = 1.0,
                 top_k: int = -1, top_p: float = 1.0, eos_id: int = -1, pad_id: int = 0, stop_check: int = 16):
        """prompts [P, Lp] int -> (sequences [P*G, Lp+max_new] int32, logp [P*G, max_new] fp32).

        top_k > 0 keeps the k most likely tokens, top_p < 1 the smallest set
        of them holding probability p (nucleus); temperature <= 0 is greedy.
        With eos_id >= 0 a sequence stops at its first eos_id (later columns
        hold pad_id and log-prob 0), ``self.last_lengths`` [P*G] gives each
        response's length (eos included) and decoding ends as soon as every
        sequence has stopped (checked every ``stop_check`` tokens)."""
        o = _ops()
        cfg, m = self.cfg, self.m
        P, Lp = prompts.shape
        G = group
        B = P * G
        if B > self.max_batch or Lp + max_new > self.max_len:
            raise ValueError("generate: batch or length beyond the engine's capacity")
        sampling = (int(top_k), float(top_p), int(eos_id), int(pad_id))
        if sampling != self.sampling:
            self.sampling = sampling
            self._graph = None  # the captured step holds the sampler's kind
        self.temperature = float(temperature)
        self.calls += 1
        table, pre_table, n_shared, tail = self._tables(P, G, Lp, max_new)
        prompts = prompts.to(self.device, torch.int32).contiguous()
        # ---- prefill the P prompts once; K/V land in the shared prompt blocks
        pos = torch.arange(Lp, device=self.device, dtype=torch.int32).repeat(P)
        seq_of_tok = torch.arange(P, device=self.device, dtype=torch.int32).repeat_interleave(Lp)
        kcs, vcs = self.kc, self.vc

        def hook(i, qkv):
            li = m.layers.index(i)
            o.kv_write(qkv, cfg.q_dim, cfg.q_dim + cfg.kv_dim, seq_of_tok, pos, pre_table, kcs[li], vcs[li],
                       cfg.n_kv_heads, cfg.head_dim, self.bs)

        x = m.embed(prompts)
        x, _ = m.forward(x, P, Lp, pos, save=False, kv_hook=hook)
        last = x.view(P, Lp, -1)[:, -1, :].contiguous()
        # a partially filled last prompt block is private: copy it to each sample's own block
        if tail:
            src_blocks = pre_table[:, n_shared].long()
            dst_blocks = table[:, n_shared].long()
            for li in range(len(m.layers)):
                kcs[li][dst_blocks] = kcs[li][src_blocks.repeat_interleave(G)]
                vcs[li][dst_blocks] = vcs[li][src_blocks.repeat_interleave(G)]
        # ---- decode state: first token sampled from the prompt's last position
        if self._graph is None or self._graph_B != (B, max_new):
            self.state = self._alloc_state(B, max_new)
            self._graph = None
        st = self.state
        st["table"].copy_(table)
        h = torch.empty(P, cfg.hidden, device=self.device, dtype=torch.bfloat16)
        o.rmsnorm_fwd(last, m.f32["norm"], h, None, cfg.rms_eps)
        hB = h.repeat_interleave(G, 0).contiguous()
        o.gemm(hB, m.head_weight(), st["logits"])
        st["step"].zero_()
        st["seed_t"].fill_(self.seed + 7919 * self.calls)
        st["temp_t"].fill_(self.temperature)
        eos = self.sampling[2] >= 0
        if eos:
            st["done"].zero_()
            st["n_done"].zero_()
            st["lengths"].fill_(max_new)
            st["tok_mat"].fill_(self.sampling[3])
            st["lp_mat"].zero_()
        self._sample(st, seed=self.seed + 7919 * self.calls + 1, temperature=self.temperature)
        o.counter_add(st["step"], 1)
        st["pos"].fill_(Lp)
        st["ctx"].fill_(Lp + 1)
        steps = max_new - 1
        if steps > 0:
            if self.cuda_graph:
                # capture one decode step once per (batch, length) shape, then
                # replay it per token; everything that changes between calls
                # (tokens, positions, block tables, seed, temperature) is read
                # from device memory
                if self._graph is None:
                    saved = {k: v.clone() for k, v in st.items() if k in ("tok", "pos", "ctx", "step")}
                    s = torch.cuda.Stream(device=self.device)
                    s.wait_stream(torch.cuda.current_stream(self.device))
                    with torch.cuda.stream(s):  # warm-up outside capture
                        self._decode_step(B)
                    torch.cuda.current_stream(self.device).wait_stream(s)
                    for k, v in saved.items():
                        st[k].copy_(v)
                    g = torch.cuda.CUDAGraph()
                    with torch.cuda.graph(g):
                        self._decode_step(B)
                    for k, v in saved.items():
                        st[k].copy_(v)
                    self._graph, self._graph_B = g, (B, max_new)
                step_fn = self._graph.replay
            else:
                def step_fn():
                    self._decode_step(B)
            done_steps = 0
            while done_steps < steps:
                n = min(stop_check if eos else steps, steps - done_steps)
                for _ in range(n):
                    step_fn()
                done_steps += n
                if eos and int(st["n_done"].item()) >= B:  # every sequence has stopped
                    break
        self.last_lengths = st["lengths"].clone() if eos else None
        seqs = torch.cat([prompts.repeat_interleave(G, 0), st["tok_mat"]], 1)
        return seqs, st["lp_mat"].clone()


# ---------------------------------------------------------------------------
@dataclass
class RolloutConfig:
    inference_backend: str = "native"  # "native" | "echo" | "vllm"
    model_path: str = ""
    tensor_parallel_size: int = 1
    max_new_tokens: int = 2048
    temperature: float = 1.0
    top_p: float = 1.0
    top_k: int = -1
    max_batch_size: int = 256
    model: str = "tiny"  # "tiny" | "qwen2-1.5b" | "llama3-8b" (random-init architectures)
    device: str = "cuda:0"
    seed: int = 0


class RolloutEngine:
    def __init__(self, config: Optional[RolloutConfig] = None):
        self.config = config or RolloutConfig()
        self.initialized = False
        self._gen: Optional[LLMGenerator] = None
        self._vllm = None
        self._tok = None

    def initialize(self):
        c = self.config
        self._tok = _core().ByteTokenizer()
        Status = _core().Status
        if c.inference_backend == "native" and torch.cuda.is_available():
            cfg = {"tiny": LMConfig.tiny(vocab=512), "qwen2-1.5b": LMConfig.qwen2_1p5b(),
                   "llama3-8b": LMConfig.llama3_8b()}[c.model]
            model = DecoderLM(cfg, c.device, seed=c.seed, master=False)
            self._gen = LLMGenerator(model, c.max_batch_size, min(cfg.max_seq, 4096), seed=c.seed)
        elif c.inference_backend == "vllm":
            from ..vllm_inference import VLLMInferenceConfig, VLLMInferenceEngine

            self._vllm = VLLMInferenceEngine(VLLMInferenceConfig(
                model=c.model_path or VLLMInferenceConfig.model, tensor_parallel_size=c.tensor_parallel_size,
                max_new_tokens=c.max_new_tokens, temperature=c.temperature, top_p=c.top_p, top_k=c.top_k,
                max_batch_size=c.max_batch_size))
        self.initialized = True
        return Status()

    def shutdown(self):
        self._gen = None
        self._vllm = None
        self.initialized = False
        return _core().Status()

    def is_native_available(self) -> bool:
        """True when generation runs on this package's own decode engine (not the echo fallback)."""
        return self._gen is not None

    def is_vllm_available(self) -> bool:
        from ..vllm_inference import vllm_available

        return vllm_available()

    def generate(self, prompt: str) -> str:
        return self.generate_batch([prompt])[0]

    def generate_batch(self, prompts: List[str]) -> List[str]:
        if not self.initialized:
            raise RuntimeError("RolloutEngine not initialized")
        if self._vllm is not None:
            return self._vllm.generate_batch(prompts)
        if self._gen is None:
            return ["[RolloutEngine] " + p for p in prompts]  # echo fallback (no GPU / no model)
        out: List[str] = []
        cap = max(1, min(self.config.max_batch_size, self._gen.max_batch))
        for i in range(0, len(prompts), cap):  # batches of at most max_batch_size prompts
            out.extend(self._generate_native(prompts[i:i + cap]))
        return out

    def _generate_native(self, prompts: List[str]) -> List[str]:
        c, tok = self.config, self._tok
        vocab = self._gen.cfg.vocab
        enc = [[t % vocab for t in tok.encode(p, True, False)] for p in prompts]
        L = max(len(e) for e in enc)
        ids = torch.full((len(enc), L), tok.pad_id % vocab, dtype=torch.int32)
        for i, e in enumerate(enc):
            ids[i, L - len(e):] = torch.tensor(e, dtype=torch.int32)  # left pad
        new = max(1, min(c.max_new_tokens, self._gen.max_len - L))
        eos = tok.eos_id % vocab
        seqs, _ = self._gen.generate(ids, 1, new, c.temperature, top_k=c.top_k, top_p=c.top_p, eos_id=eos,
                                     pad_id=tok.pad_id % vocab)
        lens = self._gen.last_lengths.cpu().tolist()
        out = seqs[:, L:].cpu().tolist()
        texts = []
        for row, n in zip(out, lens):
            row = row[:n]
            if row and row[-1] == eos:
                row = row[:-1]  # the stop token is not part of the text
            # random-init weights emit arbitrary bytes: decode leniently
            texts.append(bytes(t for t in row if t < 256).decode("utf-8", errors="replace"))
        return texts


# ---------------------------------------------------------------------------
class TPLLMGenerator(LLMGenerator):
    """LLMGenerator over a tensor-parallel model (:class:`TPDecoderLM`).

    Every rank holds the KV cache of its own KV heads for all sequences and
    runs attention for its own heads; sequences are split by rows for the
    embedding, the LM head and sampling (rank r samples sequences
    [r*B/tp, (r+1)*B/tp)).  The projections are the fused all-gather -> GEMM
    and GEMM -> reduce-scatter kernels, so the decode step (captured once as a
    CUDA graph, replayed in lockstep on all ranks) contains no NCCL call.  The
    sampled tokens are all-gathered once at the end."""

    def __init__(self, model, max_batch: int, max_len: int, block_size: int = 16, seed: int = 0,
                 cuda_graph: bool = True):
        self.tpm = model
        self.m = model.full
        self.cfg = model.cfg
        self.device = model.device
        self.max_batch, self.max_len, self.bs = max_batch, max_len, block_size
        self.seed = seed
        self.cuda_graph = cuda_graph
        self.decode_gemm = False  # the projections are the fused TP collectives
        self.blocks_per_seq = (max_len + block_size - 1) // block_size
        self.num_blocks = max_batch * self.blocks_per_seq + 1
        self.kv = _core().KVBlockManager(self.num_blocks, block_size)
        shape = (self.num_blocks, model.hk, block_size, self.cfg.head_dim)
        self.kc = [torch.empty(shape, device=self.device, dtype=torch.bfloat16) for _ in model.layers]
        self.vc = [torch.empty(shape, device=self.device, dtype=torch.bfloat16) for _ in model.layers]
        self._graph = None
        self._graph_B = None
        self.calls = 0

    def _alloc_state(self, B: int, steps: int):
        st = super()._alloc_state(B, steps)
        tpm = self.tpm
        b = B // tpm.tp
        bf = dict(device=self.device, dtype=torch.bfloat16)
        st.update({"x": torch.empty(b, self.cfg.hidden, **bf), "h": torch.empty(b, self.cfg.hidden, **bf),
                   "tok": torch.zeros(b, device=self.device, dtype=torch.int32),
                   "logits": torch.empty(b, self.cfg.vocab, **bf),
                   "tok_mat": torch.zeros(b, steps, device=self.device, dtype=torch.int32),
                   "lp_mat": torch.zeros(b, steps, device=self.device, dtype=torch.float32)})
        return st

    def _decode_step(self, B: int):
        o = _ops()
        cfg, tpm = self.cfg, self.tpm
        st = self.state
        D = cfg.head_dim
        scale = 1.0 / math.sqrt(D)
        o.embed_fwd(st["tok"], self.m.s["embed"], st["x"])
        x = st["x"]
        for li, i in enumerate(tpm.layers):
            def attn_fn(qkv, out, li=li):
                o.decode_attention(qkv, self.kc[li], self.vc[li], st["table"], st["ctx"], out, tpm.hq, tpm.hk, D,
                                   self.bs, scale)

            def hook(i_, qkv, li=li):
                o.kv_write(qkv, tpm.q_dim, tpm.q_dim + tpm.kv_dim, st["seq"], st["pos"], st["table"], self.kc[li],
                           self.vc[li], tpm.hk, D, self.bs)

            x = tpm.layer(i, x, st["pos"], B, 1, attn_fn, hook)
        o.rmsnorm_fwd(x, self.m.f32["norm"], st["h"], None, cfg.rms_eps)
        o.gemm(st["h"], self.m.head_weight(), st["logits"])
        o.sample(st["logits"], 1.0, 0, st["step"], 0, st["tok"], None, st["tok_mat"], st["lp_mat"],
                 seed_t=st["seed_t"], temp_t=st["temp_t"])
        st["pos"].add_(1)
        st["ctx"].add_(1)
        o.counter_add(st["step"], 1)

    @torch.no_grad()
    def generate(self, prompts: torch.Tensor, group: int = 1, max_new: int = 16, temperature: float = 1.0):
        """Same contract as LLMGenerator.generate; every rank passes the same
        prompts and receives the full sequences and log-probs."""
        import torch.distributed as dist

        o = _ops()
        cfg, tpm = self.cfg, self.tpm
        tp, r = tpm.tp, tpm.rank
        P, Lp = prompts.shape
        G = group
        B = P * G
        if B > self.max_batch or Lp + max_new > self.max_len:
            raise ValueError("generate: batch or length beyond the engine's capacity")
        if P % tp:
            raise ValueError("generate: the prompt count must divide by the tensor-parallel size")
        self.temperature = float(temperature)
        self.calls += 1
        table, pre_table, n_shared, tail = self._tables(P, G, Lp, max_new)
        prompts = prompts.to(self.device, torch.int32).contiguous()
        pos = torch.arange(Lp, device=self.device, dtype=torch.int32).repeat(P)
        seq_of_tok = torch.arange(P, device=self.device, dtype=torch.int32).repeat_interleave(Lp)
        kcs, vcs = self.kc, self.vc

        def hook(i, qkv):
            li = tpm.layers.index(i)
            o.kv_write(qkv, tpm.q_dim, tpm.q_dim + tpm.kv_dim, seq_of_tok, pos, pre_table, kcs[li], vcs[li],
                       tpm.hk, cfg.head_dim, self.bs)

        x = tpm.embed_rows(prompts.reshape(-1))
        x = tpm.forward(x, P, Lp, pos, kv_hook=hook)
        p_loc = P // tp
        last = x.view(p_loc, Lp, -1)[:, -1, :].contiguous()  # this rank's prompts' last positions
        if tail:
            src_blocks = pre_table[:, n_shared].long()
            dst_blocks = table[:, n_shared].long()
            for li in range(len(tpm.layers)):
                kcs[li][dst_blocks] = kcs[li][src_blocks.repeat_interleave(G)]
                vcs[li][dst_blocks] = vcs[li][src_blocks.repeat_interleave(G)]
        if self._graph is None or self._graph_B != (B, max_new):
            self.state = self._alloc_state(B, max_new)
            self._graph = None
        st = self.state
        st["table"].copy_(table)
        h = torch.empty(p_loc, cfg.hidden, device=self.device, dtype=torch.bfloat16)
        o.rmsnorm_fwd(last, self.m.f32["norm"], h, None, cfg.rms_eps)
        hB = h.repeat_interleave(G, 0).contiguous()
        o.gemm(hB, self.m.head_weight(), st["logits"])
        st["step"].zero_()
        # per-rank sampling streams: rank r samples different sequences
        st["seed_t"].fill_(self.seed + 7919 * self.calls + 104729 * r)
        st["temp_t"].fill_(self.temperature)
        o.sample(st["logits"], self.temperature, self.seed + 7919 * self.calls + 104729 * r + 1, st["step"], 0,
                 st["tok"], None, st["tok_mat"], st["lp_mat"])
        o.counter_add(st["step"], 1)
        st["pos"].fill_(Lp)
        st["ctx"].fill_(Lp + 1)
        steps = max_new - 1
        if steps > 0:
            if self.cuda_graph:
                if self._graph is None:
                    saved = {k: v.clone() for k, v in st.items() if k in ("tok", "pos", "ctx", "step")}
                    s = torch.cuda.Stream(device=self.device)
                    s.wait_stream(torch.cuda.current_stream(self.device))
                    with torch.cuda.stream(s):
                        self._decode_step(B)
                    torch.cuda.current_stream(self.device).wait_stream(s)
                    for k, v in saved.items():
                        st[k].copy_(v)
                    g = torch.cuda.CUDAGraph()
                    with torch.cuda.graph(g):
                        self._decode_step(B)
                    for k, v in saved.items():
                        st[k].copy_(v)
                    self._graph, self._graph_B = g, (B, max_new)
                for _ in range(steps):
                    self._graph.replay()
            else:
                for _ in range(steps):
                    self._decode_step(B)
        group_pg = getattr(tpm.comm, "group", None)
        tok_all = torch.empty(B, max_new, device=self.device, dtype=torch.int32)
        lp_all = torch.empty(B, max_new, device=self.device, dtype=torch.float32)
        dist.all_gather_into_tensor(tok_all, st["tok_mat"], group=group_pg)
        dist.all_gather_into_tensor(lp_all, st["lp_mat"], group=group_pg)
        seqs = torch.cat([prompts.repeat_interleave(G, 0), tok_all], 1)
        return seqs, lp_all
