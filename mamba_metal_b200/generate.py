"""Autoregressive generation -- drop-in for mamba_metal/generate.py:16-110, plus a batched id-level
driver.

- ``generate``      : O(L^2), re-runs the full forward each step (generate.py:16-62).
- ``generate_fast`` : O(L), one parallel prefill then ``model.step`` per token with the carried conv and
  SSM state (generate.py:65-110). Greedy ties resolve to the first maximal index, as mx.argmax.
- ``generate_ids``  : the same prefill -> decode hand-off for a (B, L) batch of token ids without a
  tokenizer (the reference's generate_fast is batch-1 by construction, generate.py:94, :106). The
  decode step, greedy argmax included, is captured once in a CUDA graph and replayed per token with the
  state tensors updated in place; the host synchronises once at the end.
"""

from __future__ import annotations

from typing import Callable

import numpy as np
import torch


def _ids_tensor(tokenizer, prompt: str, device) -> torch.Tensor:
    ids = tokenizer(prompt, return_tensors="np").input_ids
    return torch.as_tensor(np.asarray(ids), dtype=torch.long, device=device)


def _pick(next_logits: torch.Tensor, temperature: float) -> torch.Tensor:
    if temperature == 0.0:
        return torch.argmax(next_logits, dim=-1)
    probs = torch.softmax(next_logits.float() / temperature, dim=-1)
    return torch.multinomial(probs, 1)[:, 0]


def _stream(on_token, tokenizer, generated, prompt, prev_text):
    if on_token is None:
        return prev_text
    new_text = tokenizer.decode(generated, skip_special_tokens=True)
    delta = new_text[len(prev_text) - len(prompt):]
    if delta:
        on_token(delta)
        prev_text = prompt + new_text
    return prev_text


@torch.no_grad()
def generate(model, tokenizer, prompt: str, max_new_tokens: int = 50, temperature: float = 0.0,
             on_token: Callable[[str], None] | None = None) -> str:
    """O(L^2) generation: full forward per token (generate.py:16-62)."""
    device = model.embeddings.weight.device
    input_ids = _ids_tensor(tokenizer, prompt, device)
    eos = tokenizer.eos_token_id
    generated: list[int] = []
    prev_text = prompt
    for _ in range(max_new_tokens):
        next_logits = model(input_ids)[:, -1, :]
        nid = int(_pick(next_logits, temperature)[0].item())
        if eos is not None and nid == eos:
            break
        generated.append(nid)
        prev_text = _stream(on_token, tokenizer, generated, prompt, prev_text)
        input_ids = torch.cat([input_ids, torch.tensor([[nid]], dtype=input_ids.dtype, device=device)], dim=1)
    return prompt + tokenizer.decode(generated, skip_special_tokens=True)


@torch.no_grad()
def generate_fast(model, tokenizer, prompt: str, max_new_tokens: int = 50, temperature: float = 0.0,
                  on_token: Callable[[str], None] | None = None) -> str:
    """O(L_prompt + n_decode) generation: parallel prefill, then O(1) per token (generate.py:65-110)."""
    device = model.embeddings.weight.device
    input_ids = _ids_tensor(tokenizer, prompt, device)
    eos = tokenizer.eos_token_id
    logits, conv_states, ssm_states = model.prefill(input_ids, last_only=True)
    next_logits = logits[:, -1, :]
    generated: list[int] = []
    prev_text = prompt
    for _ in range(max_new_tokens):
        nid = int(_pick(next_logits, temperature)[0].item())
        if eos is not None and nid == eos:
            break
        generated.append(nid)
        prev_text = _stream(on_token, tokenizer, generated, prompt, prev_text)
        ids = torch.tensor([[nid]], dtype=torch.long, device=device)
        step_logits, conv_states, ssm_states = model.step(ids, conv_states, ssm_states, inplace=True)
        next_logits = step_logits[:, 0, :]
    return prompt + tokenizer.decode(generated, skip_special_tokens=True)


class GraphDecoder:
    """Greedy decode step captured in one CUDA graph: ids (B, 1) -> model.step (states in place) ->
    argmax -> ids. Replaying it advances every sequence by one token without host synchronisation."""

    def __init__(self, model, conv_states, ssm_states, first_ids: torch.Tensor):
        self.model = model
        self.conv_states, self.ssm_states = conv_states, ssm_states
        self.ids = first_ids.reshape(-1, 1).to(torch.long).clone()
        self.logits = None
        # warm up on copies so that lazy initialisation (cuBLAS handles, module loading) happens outside
        # the capture without advancing the real state
        side = torch.cuda.Stream(device=self.ids.device)
        side.wait_stream(torch.cuda.current_stream(self.ids.device))
        with torch.cuda.stream(side):
            cs = [c.clone() for c in conv_states]
            ss = [s.clone() for s in ssm_states]
            for _ in range(2):
                lg, _, _ = model.step(self.ids, cs, ss, inplace=True)
                torch.argmax(lg[:, 0, :], dim=-1)
        torch.cuda.current_stream(self.ids.device).wait_stream(side)
        del cs, ss
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph):
            lg, _, _ = model.step(self.ids, self.conv_states, self.ssm_states, inplace=True)
            self.logits = lg
            self.ids.copy_(torch.argmax(lg[:, 0, :], dim=-1, keepdim=True))

    def step(self) -> torch.Tensor:
        """Consumes self.ids, produces the next ids (in self.ids) and returns them."""
        self.graph.replay()
        return self.ids


@torch.no_grad()
def generate_ids(model, input_ids: torch.Tensor, max_new_tokens: int, temperature: float = 0.0,
                 use_graph: bool = True) -> torch.Tensor:
    """Batched prefill -> decode on token ids (B, L). Returns (B, max_new_tokens) generated ids.

    Greedy decoding uses the CUDA-graph step; sampling (temperature > 0) runs eagerly."""
    logits, conv_states, ssm_states = model.prefill(input_ids, last_only=True)
    first = _pick(logits[:, -1, :], temperature)
    out = torch.empty((input_ids.shape[0], max_new_tokens), dtype=torch.long, device=input_ids.device)
    if max_new_tokens == 0:
        return out
    out[:, 0] = first
    if temperature == 0.0 and use_graph:
        dec = GraphDecoder(model, conv_states, ssm_states, first)
        for i in range(1, max_new_tokens):
            out[:, i] = dec.step()[:, 0]
        return out
    ids = first[:, None]
    for i in range(1, max_new_tokens):
        lg, conv_states, ssm_states = model.step(ids, conv_states, ssm_states, inplace=True)
        ids = _pick(lg[:, 0, :], temperature)[:, None]
        out[:, i] = ids[:, 0]
    return out
