"""EAGLE3 draft head (Llama-3 family) and its proposer.

Draft model (the EAGLE3 checkpoint layout: ``fc``, ``midlayer.*``, ``norm``, ``lm_head``,
``d2t``): the target's hidden states after three layers (low / middle / high) are fused by
``fc [H, 3H]``; one decoder layer whose attention input is ``[input_norm(embed(token)) ||
hidden_norm(hidden)]`` (2H wide), a SwiGLU MLP, a final norm and a draft-vocabulary LM head whose
ids map to target ids by ``target = draft + d2t[draft]``.  Draft step 1 consumes the fused
target states; later steps feed back the draft layer's own output state.

The draft attends over a window of the most recent ``window`` positions of each request
(recomputed every step from the stored target states), so it needs no KV cache of its own; a
full-context draft would accept more drafts on real checkpoints, but every emitted token is
verified by the target model either way, so the window only affects speed, never output.

Reference: vllm_neuron/vllm/spec_decode/eagle.py:32-512 (EagleProposer.propose :404) and
vllm_neuron/model/llama3/eagle3_model.py (draft layer, FC fusion of the three aux states).
"""
from __future__ import annotations

import json
import math
import os

import torch
import torch.nn.functional as F

from ..ops.rope import apply_rope_ref


def default_aux_layers(num_layers: int) -> list[int]:
    return [2, num_layers // 2, num_layers - 3]


class Eagle3Draft(torch.nn.Module):
    def __init__(self, H: int, Hq: int, Hkv: int, D: int, I: int, V_draft: int, eps: float, device, dtype):
        super().__init__()
        self.H, self.Hq, self.Hkv, self.D, self.I, self.eps = H, Hq, Hkv, D, I, eps
        p = lambda *s: torch.nn.Parameter(torch.empty(*s, dtype=dtype, device=device), requires_grad=False)
        self.fc = p(H, 3 * H)
        self.input_norm = p(H)
        self.hidden_norm = p(H)
        self.qkv = p((Hq + 2 * Hkv) * D, 2 * H)
        self.o = p(H, Hq * D)
        self.post_norm = p(H)
        self.gate_up = p(2 * I, H)
        self.down = p(H, I)
        self.norm = p(H)
        self.lm_head = p(V_draft, H)
        self.register_buffer("d2t", torch.zeros(V_draft, dtype=torch.int64, device=device))

    def _rms(self, x, w):
        xf = x.float()
        return (xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + self.eps) * w.float()).to(x.dtype)

    @torch.no_grad()
    def forward(self, emb: torch.Tensor, hidden: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor):
        """``emb, hidden [W, H]`` (hidden already fused), ``cos/sin [W, rot/2]`` -> (output
        hidden state [W, H] before the final norm, logits of the last row [V_draft])."""
        W = emb.shape[0]
        residual = hidden
        x = torch.cat([self._rms(emb, self.input_norm), self._rms(hidden, self.hidden_norm)], -1)
        qkv = (x @ self.qkv.t()).float()
        q = qkv[:, :self.Hq * self.D].view(W, self.Hq, self.D)
        k = qkv[:, self.Hq * self.D:(self.Hq + self.Hkv) * self.D].view(W, self.Hkv, self.D)
        v = qkv[:, (self.Hq + self.Hkv) * self.D:].view(W, self.Hkv, self.D)
        q = apply_rope_ref(q, cos, sin, True)
        k = apply_rope_ref(k, cos, sin, True)
        g = self.Hq // self.Hkv
        k = k.repeat_interleave(g, 1)
        v = v.repeat_interleave(g, 1)
        s = torch.einsum("qhd,khd->hqk", q, k) / math.sqrt(self.D)
        mask = torch.ones(W, W, dtype=torch.bool, device=s.device).tril()
        s = s.masked_fill(~mask, float("-inf"))
        a = torch.einsum("hqk,khd->qhd", torch.softmax(s, -1), v).reshape(W, -1).to(emb.dtype)
        h = a @ self.o.t() + residual
        y = self._rms(h, self.post_norm)
        gu = y @ self.gate_up.t()
        y = (F.silu(gu[:, :self.I].float()) * gu[:, self.I:].float()).to(emb.dtype) @ self.down.t()
        out = h + y
        logits = self._rms(out[-1:], self.norm) @ self.lm_head.t()
        return out, logits[0]


class Eagle3Proposer:
    """Drafts k tokens per decoding request with an :class:`Eagle3Draft` over a window of
    recent positions; the target model exports its aux hidden states every step."""

    def __init__(self, engine, cfg: dict, k: int):
        self.engine = engine
        self.k = k
        self.window = int(cfg.get("window", 32))
        m = engine.model
        tc = m.cfg
        self.aux_layers = list(cfg.get("aux_layers") or default_aux_layers(tc.num_layers))
        m.enable_aux_hidden(self.aux_layers)
        path = cfg.get("model")
        dcfg = {}
        if path and os.path.isfile(os.path.join(path, "config.json")):
            dcfg = json.load(open(os.path.join(path, "config.json")))
        H = tc.hidden_size
        Hq, Hkv, D = tc.num_heads, tc.num_kv_heads, tc.head_dim
        I = dcfg.get("intermediate_size", tc.intermediate_size)
        Vd = dcfg.get("draft_vocab_size", tc.vocab_size)
        self.draft = Eagle3Draft(H, Hq, Hkv, D, I, Vd, tc.rms_norm_eps, m.device, m.dtype)
        if path:
            self._load(path)
        else:
            self._random_init(int(cfg.get("seed", 0)))
        self.cos_sin = m.cos_sin.to(m.device)
        self.rot = tc.rot_dim
        self.hist: dict[str, tuple[torch.Tensor, list[int]]] = {}  # req -> (aux [n, 3H], positions)

    @torch.no_grad()
    def _random_init(self, seed: int):
        g = torch.Generator(device=self.draft.fc.device)
        g.manual_seed(seed)
        for n, prm in self.draft.named_parameters():
            if "norm" in n:
                prm.fill_(1.0)
            else:
                prm.normal_(0.0, 0.02, generator=g)

    @torch.no_grad()
    def _load(self, path: str):
        from ..utils.checkpoints import SafetensorsCheckpoint

        ck = SafetensorsCheckpoint(path)
        names = ck.names()
        get = lambda n: ck.get(n).to(self.draft.fc.device)  # noqa: E731
        pre = "midlayer." if any(n.startswith("midlayer.") for n in names) else "layers.0."
        d = self.draft
        d.fc.copy_(get("fc.weight"))
        d.input_norm.copy_(get(pre + "input_layernorm.weight"))
        d.hidden_norm.copy_(get(pre + "hidden_norm.weight"))
        d.qkv.copy_(torch.cat([get(pre + f"self_attn.{x}_proj.weight") for x in "qkv"], 0))
        d.o.copy_(get(pre + "self_attn.o_proj.weight"))
        d.post_norm.copy_(get(pre + "post_attention_layernorm.weight"))
        d.gate_up.copy_(torch.cat([get(pre + "mlp.gate_proj.weight"), get(pre + "mlp.up_proj.weight")], 0))
        d.down.copy_(get(pre + "mlp.down_proj.weight"))
        d.norm.copy_(get("norm.weight"))
        d.lm_head.copy_(get("lm_head.weight"))
        if "d2t" in names:
            d.d2t.copy_(get("d2t").long())

    def _embed(self, toks: list[int]) -> torch.Tensor:
        m = self.engine.model
        ids = torch.tensor(toks, dtype=torch.long, device=m.device)
        # the target's (vocab-sharded) embedding; drafts run replicated on every rank
        e = m.embed
        if m.tp.world == 1:
            return e[ids]
        local = ids - m.vocab_start
        ok = (local >= 0) & (local < m.V_local)
        out = torch.where(ok[:, None], e[local.clamp(0, m.V_local - 1)], torch.zeros((), dtype=e.dtype, device=e.device))
        return m.tp.all_reduce_(out)

    def observe(self, out, accepted: list[list[int]]):
        """Store the target's aux states of the positions this step made valid."""
        m = self.engine.model
        t = 0
        k = 0
        for sr in out.scheduled:
            n = sr.num_tokens
            rows = m.aux_hidden[t:t + n]
            valid = n
            if sr.samples:
                if sr.spec:
                    valid = len(accepted[k])  # last token + accepted drafts
                k += 1
            rid = sr.req.request_id
            if sr.start == 0:  # (re)computation from the start: forget older states
                self.hist.pop(rid, None)
            aux, pos = self.hist.get(rid, (rows[:0], []))
            aux = torch.cat([aux, rows[:valid]], 0)[-self.window:]
            pos = (pos + list(range(sr.start, sr.start + valid)))[-self.window:]
            self.hist[rid] = (aux.clone(), pos)
            t += n

    @torch.no_grad()
    def propose(self, requests) -> dict[str, list[int]]:
        res = {}
        d = self.draft
        for r in requests:
            h = self.hist.get(r.request_id)
            if h is None or not len(h[1]):
                res[r.request_id] = []
                continue
            aux, pos = h
            toks_all = r.all_token_ids()
            # pair (token at p + 1, target state at p)
            nxt = [toks_all[p + 1] for p in pos]
            hidden = aux @ d.fc.t()
            positions = list(pos)
            draft = []
            for _ in range(self.k):
                cs = self.cos_sin[torch.tensor(positions, device=aux.device)]
                half = self.rot // 2
                out, logits = d(self._embed(nxt), hidden, cs[:, :half], cs[:, half:self.rot])
                di = int(logits.argmax())
                tok = di + int(d.d2t[di])
                draft.append(tok)
                nxt = nxt + [tok]
                hidden = torch.cat([hidden, out[-1:]], 0)
                positions = positions + [positions[-1] + 1]
            res[r.request_id] = draft
        return res

    def release(self, request_id: str):
        self.hist.pop(request_id, None)
