"""CUDA-graph prefill and whole-step decode drivers for ESAModel.

The reference decode loop (esa/model.py:1007-1072) does, per token, a host
tensor for the position (an H2D copy), ~10 launches per layer, a
``states.clone()`` and a host-side sampling call.  Here one decode step --
embedding + position, every layer's qgv GEMV, the fused Lightning kernel,
out_proj, MLP, lm_head, the greedy argmax, and the bookkeeping (state
write-back, position advance modulo ``block``, output slot) -- is captured once
in a CUDA graph over static buffers and replayed per token with no host work.

Greedy decoding (temperature <= 0) runs entirely on the device.  With
temperature > 0 the logits are captured and sampling runs with
``sample_next_token`` on the current stream after each replay (still no host
synchronisation).  EOS handling: all steps are replayed, then the sequence is
cut after the first step at which every row produced ``eos_token_id``, which is
what the reference's early exit returns.
"""

from __future__ import annotations

import torch

from .generation import sample_next_token


class DecodeGraph:
    def __init__(self, model, batch: int, state_dtype: torch.dtype, *, temperature: float = 0.0,
                 top_k=None, top_p=None, warmup: int = 2):
        cfg = model.config
        dev = model.device
        self.model = model
        self.block = int(cfg.block)
        self.greedy = float(temperature) <= 0
        self.temperature, self.top_k, self.top_p = temperature, top_k, top_p
        H, D = cfg.head, cfg.embd // cfg.head
        self.token = torch.zeros(batch, dtype=torch.long, device=dev)
        self.states = torch.zeros(cfg.n_layer, batch, H, D, dtype=state_dtype, device=dev)
        self.pos = torch.zeros((), dtype=torch.long, device=dev)
        self.graph = None
        self._warmup = warmup
        self.logits = None

    def _step(self):
        logits, new_states = self.model.lightning_step(self.token, self.states, self.pos)
        self.states.copy_(new_states)
        self.pos.add_(1).remainder_(self.block)
        if self.greedy:
            self.token.copy_(torch.argmax(logits, dim=-1))
        return logits

    def _capture(self):
        s = torch.cuda.Stream(device=self.token.device)
        s.wait_stream(torch.cuda.current_stream())
        saved = (self.token.clone(), self.states.clone(), self.pos.clone())
        with torch.cuda.stream(s):
            for _ in range(self._warmup):
                self._step()
        torch.cuda.current_stream().wait_stream(s)
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph):
            self.logits = self._step()
        self.token.copy_(saved[0])
        self.states.copy_(saved[1])
        self.pos.copy_(saved[2])

    @torch.inference_mode()
    def run(self, first_token: torch.Tensor, states: torch.Tensor, prefill_len: int, steps: int, *,
            eos_token_id=None) -> torch.Tensor:
        """Decode `steps` tokens after `first_token`; returns [B, 1 + steps'] ids."""
        if self.graph is None:
            self._capture()
        self.token.copy_(first_token.reshape(-1))
        self.states.copy_(states)
        self.pos.fill_(int(prefill_len) % self.block)
        out = torch.empty(self.token.numel(), steps + 1, dtype=torch.long, device=self.token.device)
        out[:, 0] = self.token
        for i in range(steps):
            self.graph.replay()
            if not self.greedy:
                nxt = sample_next_token(self.logits, temperature=self.temperature, top_k=self.top_k,
                                        top_p=self.top_p)
                self.token.copy_(nxt.reshape(-1))
            out[:, i + 1] = self.token
        if eos_token_id is not None:
            hit = (out[:, 1:] == int(eos_token_id)).all(dim=0)
            idx = torch.nonzero(hit)
            if idx.numel():
                out = out[:, : int(idx[0]) + 2]
        return out


class PrefillGraph:
    """The prompt prefill of a fixed [B, T] (embedding, every block's ESA
    prefill and MLP, the last position's logits and the states), captured once
    in a CUDA graph and replayed per call: the eager prefill of a short prompt
    spends most of its time launching a few hundred small kernels from the
    host.  Outputs are the graph's static buffers, overwritten by the next
    replay (copy what must outlive it)."""

    def __init__(self, model, shape, backend, compass, warmup: int = 2):
        self.model = model
        self.backend, self.compass = backend, compass
        self.ids = torch.zeros(shape, dtype=torch.long, device=model.device)
        self.graph = None
        self.out = None
        self._warmup = warmup

    def _capture(self):
        s = torch.cuda.Stream(device=self.ids.device)
        s.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(s):
            for _ in range(self._warmup):
                self.model._prefill_eager(self.ids, backend=self.backend, compass=self.compass)
        torch.cuda.current_stream().wait_stream(s)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            self.out = self.model._prefill_eager(self.ids, backend=self.backend, compass=self.compass)
        self.graph = graph

    @torch.inference_mode()
    def run(self, input_ids: torch.Tensor):
        """(logits [B, V], states, T) of the prompt, as _prefill_eager."""
        self.ids.copy_(input_ids)
        if self.graph is None:
            self._capture()
        self.graph.replay()
        return self.out
