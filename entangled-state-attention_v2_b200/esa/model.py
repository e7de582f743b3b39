# Copyright 2026 Zameer Hussain and Akhtar Hussain
# Licensed under the Apache License, Version 2.0.
# Portions of this file reproduce the public interface of esa/model.py of
# Entangled-State-Attention v2.1.1 (signatures, dataclasses, validation and
# error messages), under that licence.

"""ESAModel: the causal LM driver of the ESA layers (reference esa/model.py).

Same configuration dataclass, module tree, parameter names (state_dict keys),
initialisation, forward / prefill / lightning_step / generate / save / load
behaviour as the reference (esa/model.py:58-1256).  The ESA layers run the B200
scan kernels; LayerNorm, MLP, embeddings and lm_head stay on cuBLAS / ATen.

Decode driver: with ``compile=True`` the reference wraps ``lightning_step`` in
``torch.compile``; here the whole step (all layers, the fused Lightning kernel,
lm_head and the greedy/sampling head) can instead be captured once in a CUDA
graph (``runtime="lightning_graph"`` or ``decode_graph=True``), removing the
per-token launch overhead.  The default follows the reference.
"""

from __future__ import annotations

import importlib.util
import json
import math
import time
import warnings
from dataclasses import asdict, dataclass
from pathlib import Path
from typing import Any

import torch
import torch.nn as nn
import torch.nn.functional as F

from . import ops
from .generation import GenerationResult, GenerationStats, parse_engine_spec, sample_next_token
from .layer import ESA


def available_devices() -> dict[str, bool]:
    """Devices ESA knows about (only CUDA runs the ESA kernels in this build)."""
    return {
        "cpu": True,
        "cuda": torch.cuda.is_available(),
        "mps": hasattr(torch.backends, "mps") and torch.backends.mps.is_available(),
        "xla": importlib.util.find_spec("torch_xla") is not None,
        "npu": importlib.util.find_spec("torch_npu") is not None,
    }


def print_available_devices() -> None:
    devices = available_devices()
    print("\nAvailable Devices\n-----------------------------")
    for name, enabled in devices.items():
        print(f"{'✓' if enabled else '✗'} {name}")
    if devices["cuda"]:
        print(f"\nCUDA GPU : {torch.cuda.get_device_name(0)}")


@dataclass
class ESAModelConfig:
    vocab_size: int
    block: int = 512
    n_layer: int = 6
    head: int = 6
    embd: int = 384
    dropout: float = 0.1
    bias: bool = True
    backend: str = "thunder"
    precision: str = "fp16"
    compass: int | None = None
    training_compile: bool = True
    training_compile_mode: str = "default"
    training_compile_fullgraph: bool = False
    gate_min: float = 0.80
    gate_max: float = 0.995
    eps: float = 1e-5
    tie_embeddings: bool = True
    format_version: int = 1

    @classmethod
    def from_dict(cls, data: dict[str, Any]) -> "ESAModelConfig":
        """Construct a configuration from a dict, ignoring unknown keys."""
        allowed = cls.__dataclass_fields__.keys()
        return cls(**{k: v for k, v in data.items() if k in allowed})


class _LayerNorm(nn.Module):
    def __init__(self, ndim: int, bias: bool):
        super().__init__()
        self.weight = nn.Parameter(torch.ones(ndim))
        self.bias = nn.Parameter(torch.zeros(ndim)) if bias else None

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        # On the GPU: the fused kernel, writing the dtype the consuming Linear
        # computes in (the autocast dtype under autocast; the same values as an
        # fp32 result cast by the Linear).  Elsewhere (no bias, fp64, odd
        # widths): F.layer_norm.
        if ops.layer_norm_supported(x, self.weight, self.bias):
            out_dtype = x.dtype
            if torch.is_autocast_enabled("cuda"):
                out_dtype = torch.get_autocast_dtype("cuda")
            y, _, _ = ops.layer_norm(x, self.weight, self.bias, 1e-5, out_dtype)
            return y
        return F.layer_norm(x, self.weight.shape, self.weight, self.bias, 1e-5)

    def add_forward(self, x: torch.Tensor, res: torch.Tensor):
        """(x + res, LayerNorm(x + res)): the residual add and the norm after it,
        one fused kernel on the GPU (the sum in x's dtype, as `x + res`)."""
        if (ops.layer_norm_supported(x, self.weight, self.bias) and res.is_cuda
                and res.shape == x.shape and torch.result_type(x, res) == x.dtype
                and res.dtype in (torch.float16, torch.bfloat16, torch.float32)):
            out_dtype = x.dtype
            if torch.is_autocast_enabled("cuda"):
                out_dtype = torch.get_autocast_dtype("cuda")
            xsum, y, _, _ = ops.add_layer_norm(x, res, self.weight, self.bias, 1e-5, out_dtype)
            return xsum, y
        x = x + res
        return x, self(x)


class _MLP(nn.Module):
    def __init__(self, cfg: ESAModelConfig):
        super().__init__()
        self.fc = nn.Linear(cfg.embd, 4 * cfg.embd, bias=cfg.bias)
        self.proj = nn.Linear(4 * cfg.embd, cfg.embd, bias=cfg.bias)
        self.drop = nn.Dropout(cfg.dropout)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        return self.drop(self.proj(F.gelu(self.fc(x))))


class _ESABlock(nn.Module):
    def __init__(self, cfg: ESAModelConfig):
        super().__init__()
        self.ln1 = _LayerNorm(cfg.embd, cfg.bias)
        self.esa = ESA(embd=cfg.embd, head=cfg.head, block=cfg.block, backend=cfg.backend,
                       precision=cfg.precision, compass=cfg.compass, dropout=cfg.dropout,
                       gate_min=cfg.gate_min, gate_max=cfg.gate_max, eps=cfg.eps, device=None)
        self.ln2 = _LayerNorm(cfg.embd, cfg.bias)
        self.mlp = _MLP(cfg)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        x, h = self.ln2.add_forward(x, self.esa(self.ln1(x)))
        return x + self.mlp(h)

    def fused_forward(self, x: torch.Tensor, pending: torch.Tensor | None):
        """forward(x + pending) returned as (x', pending'): the block's residual
        adds fused into the norms after them.  `pending` is the previous
        block's MLP output not yet added to x; the caller adds the last one."""
        if pending is None:
            h = self.ln1(x)
        else:
            x, h = self.ln1.add_forward(x, pending)
        x, h = self.ln2.add_forward(x, self.esa(h))
        return x, self.mlp(h)

    @torch.no_grad()
    def prefill(self, x: torch.Tensor, *, backend: str | None = None, compass: int | None = None):
        y, state = self.esa.prefill(self.ln1(x), backend=backend, compass=compass)
        x = x + y
        return x + self.mlp(self.ln2(x)), state

    lightning_prefill = prefill

    def lightning_step(self, x: torch.Tensor, state: torch.Tensor):
        y, new_state = self.esa.decode_step(self.ln1(x), state)
        x, h = self.ln2.add_forward(x, y)
        return x + self.mlp(h), new_state

    def fused_lightning_step(self, x: torch.Tensor, pending: torch.Tensor | None, state: torch.Tensor):
        """lightning_step(x + pending) as (x', pending', new state), the residual
        adds fused into the norms (see fused_forward).  A few rows of a 16-bit
        model run the whole block in four fused launches (ops.decode_block)."""
        if ops.decode_block_supported(x, self):
            from .generation import _unwrap_backend
            bk = _unwrap_backend(self.esa)
            return ops.decode_block(x, pending, state, self, bk.gate_min, bk.gate_max, bk.eps, bk.qgv,
                                    bk.out_proj)
        if pending is None:
            h = self.ln1(x)
        else:
            x, h = self.ln1.add_forward(x, pending)
        y, new_state = self.esa.decode_step(h, state)
        x, h = self.ln2.add_forward(x, y)
        return x, self.mlp(h), new_state


def _resolve_device(device) -> torch.device:
    name = str(device).lower()
    if name == "cuda":
        if torch.cuda.is_available():
            return torch.device("cuda")
        warnings.warn("CUDA requested but not available. Falling back to CPU.", RuntimeWarning,
                      stacklevel=3)
        return torch.device("cpu")
    if name == "cpu":
        return torch.device("cpu")
    if name.startswith("cuda:"):
        return torch.device(name)
    if name == "mps":
        if hasattr(torch.backends, "mps") and torch.backends.mps.is_available():
            return torch.device("mps")
        raise RuntimeError("MPS requested but Apple MPS is not available.")
    if name in {"tpu", "xla"}:
        try:
            import torch_xla.core.xla_model as xm
        except ImportError as exc:
            raise RuntimeError("TPU/XLA requested but torch_xla is not installed.") from exc
        return xm.xla_device()
    if name == "npu":
        try:
            import torch_npu  # noqa: F401
        except ImportError as exc:
            raise RuntimeError("NPU requested but torch_npu is not installed.") from exc
        return torch.device("npu")
    raise ValueError(f"Unsupported ESA device: {device!r}. "
                     "Choose from: 'cuda', 'cpu', 'mps', 'tpu', 'xla', or 'npu'.")


class ESAModel(nn.Module):
    """Causal language model built from ESA layers.

    Lifecycle: model(...), model.generate(...), model.save(...), ESAModel.load(...).
    """

    def __init__(self, config: ESAModelConfig | None = None, *, device: str = "cuda", **kwargs: Any):
        super().__init__()
        if config is None:
            config = ESAModelConfig(**kwargs)
        elif kwargs:
            raise TypeError("Pass either config=... or keyword configuration, not both.")
        self.config = config
        target = _resolve_device(device)

        self.wte = nn.Embedding(config.vocab_size, config.embd)
        self.wpe = nn.Embedding(config.block, config.embd)
        self.drop = nn.Dropout(config.dropout)
        self.blocks = nn.ModuleList([_ESABlock(config) for _ in range(config.n_layer)])
        self.ln_f = _LayerNorm(config.embd, config.bias)
        self.lm_head = nn.Linear(config.embd, config.vocab_size, bias=False)
        if config.tie_embeddings:
            self.wte.weight = self.lm_head.weight
        self.apply(self._init_weights)
        for name, p in self.named_parameters():
            if name.endswith(("proj.weight", "out_proj.weight")) and p.ndim >= 2:
                nn.init.normal_(p, mean=0.0, std=0.02 / math.sqrt(2 * config.n_layer))

        self._compiled_lightning_step = None
        self._compiled_lightning_key = None
        self._compiled_prefill_cache: dict[tuple[Any, ...], Any] = {}
        self._prefill_compile_failures: set[tuple[Any, ...]] = set()
        self._compiled_training_forward = None
        self._compiled_training_key = None
        self._training_compile_failed = False
        self._compile_warnings_emitted: set[str] = set()
        self._decode_graphs: dict[tuple[Any, ...], Any] = {}
        self._prefill_graphs: dict[tuple[Any, ...], Any] = {}
        self._prefill_graph_failures: set[tuple[Any, ...]] = set()
        self.to(target)

    def _init_weights(self, module: nn.Module) -> None:
        if isinstance(module, nn.Linear):
            nn.init.normal_(module.weight, mean=0.0, std=0.02)
            if module.bias is not None:
                nn.init.zeros_(module.bias)
        elif isinstance(module, nn.Embedding):
            nn.init.normal_(module.weight, mean=0.0, std=0.02)

    @property
    def device(self) -> torch.device:
        return self.wte.weight.device

    # ------------------------------------------------------------------ training
    def _forward_eager(self, input_ids: torch.Tensor, targets: torch.Tensor | None = None):
        _, T = input_ids.shape
        if T > self.config.block:
            raise ValueError(f"Sequence length {T} exceeds block {self.config.block}.")
        pos = torch.arange(T, dtype=torch.long, device=input_ids.device)
        x = self.drop(self.wte(input_ids) + self.wpe(pos)[None, :, :])
        pending = None
        for block in self.blocks:
            x, pending = block.fused_forward(x, pending)
        h = self.ln_f(x) if pending is None else self.ln_f.add_forward(x, pending)[1]
        logits = self.lm_head(h)
        loss = None
        if targets is not None:
            flat, tflat = logits.reshape(-1, logits.size(-1)), targets.reshape(-1)
            if ops.cross_entropy_supported(flat, tflat):
                # fused LM-head loss: reads the 16-bit logits twice in all,
                # instead of an fp32 copy, an fp32 log-softmax and their backward
                loss = ops.cross_entropy(flat, tflat, ignore_index=-1)
            else:
                loss = F.cross_entropy(flat, tflat, ignore_index=-1)
        return logits, loss

    def compile_training(self, *, mode: str | None = None, fullgraph: bool | None = None) -> "ESAModel":
        """Compile the full training forward (ESA kernels are opaque custom ops)."""
        if not hasattr(torch, "compile"):
            return self
        mode = mode or self.config.training_compile_mode
        fullgraph = self.config.training_compile_fullgraph if fullgraph is None else bool(fullgraph)
        key = (mode, fullgraph)
        if self._compiled_training_key == key and self._compiled_training_forward is not None:
            return self
        try:
            self._compiled_training_forward = torch.compile(self._forward_eager, mode=mode,
                                                            fullgraph=fullgraph)
            self._compiled_training_key = key
            self._training_compile_failed = False
        except Exception as exc:
            self._compiled_training_forward = None
            self._training_compile_failed = True
            self._warn_compile_fallback("training", exc)
        return self

    def forward(self, input_ids: torch.Tensor, targets: torch.Tensor | None = None):
        use_compiled = (bool(self.config.training_compile) and self.device.type == "cuda"
                        and self.training and targets is not None
                        and not self._training_compile_failed)
        if use_compiled:
            if self._compiled_training_forward is None:
                self.compile_training()
            if self._compiled_training_forward is not None:
                return self._compiled_training_forward(input_ids, targets)
        return self._forward_eager(input_ids, targets)

    # ------------------------------------------------------------------ prefill
    @torch.no_grad()
    def _prefill_eager(self, input_ids: torch.Tensor, *, backend: str | None = None,
                       compass: int | None = None):
        if input_ids.ndim != 2:
            raise ValueError(f"input_ids must be [B,T], got {tuple(input_ids.shape)}")
        if input_ids.size(1) > self.config.block:
            input_ids = input_ids[:, -self.config.block:]
        T = input_ids.size(1)
        if T <= 0:
            raise ValueError("Prefill requires at least one token.")
        pos = torch.arange(T, device=input_ids.device)
        x = self.drop(self.wte(input_ids) + self.wpe(pos)[None, :, :])
        states = []
        for block in self.blocks:
            x, state = block.prefill(x, backend=backend, compass=compass)
            states.append(state)
        states_out = torch.stack(states, dim=0).contiguous()
        logits = self.lm_head(self.ln_f(x[:, -1]))
        return logits, states_out, T

    def _warn_compile_fallback(self, component: str, exc: Exception) -> None:
        if component in self._compile_warnings_emitted:
            return
        self._compile_warnings_emitted.add(component)
        warnings.warn(f"ESA {component} compilation failed; falling back to eager execution: {exc}",
                      RuntimeWarning, stacklevel=2)

    def _cudagraph_mark_step_begin(self) -> None:
        if self.device.type != "cuda":
            return
        marker = getattr(getattr(torch, "compiler", None), "cudagraph_mark_step_begin", None)
        if marker is not None:
            marker()

    @torch.no_grad()
    def prefill(self, input_ids: torch.Tensor, *, engine: str = "thunder_compiled_16",
                compile_mode: str = "default", fullgraph: bool = False, dynamic: bool = True):
        """Prompt prefill with a selectable engine; returns (logits, states, T)."""
        spec = parse_engine_spec(engine)

        def eager(ids):
            return self._prefill_eager(ids, backend=spec.backend, compass=spec.compass)

        if spec.compiled and self.device.type == "cuda" and hasattr(torch, "compile"):
            key = (spec.backend, spec.compass, bool(fullgraph), bool(dynamic), False)
            fn = self._compiled_prefill_cache.get(key)
            if fn is None and key not in self._prefill_compile_failures:
                try:
                    fn = torch.compile(eager, fullgraph=fullgraph, dynamic=True,
                                       options={"triton.cudagraphs": False})
                    self._compiled_prefill_cache[key] = fn
                except Exception as exc:
                    self._prefill_compile_failures.add(key)
                    self._warn_compile_fallback("prefill", exc)
            if fn is not None:
                try:
                    return fn(input_ids)
                except Exception as exc:
                    self._prefill_compile_failures.add(key)
                    self._compiled_prefill_cache.pop(key, None)
                    self._warn_compile_fallback("prefill", exc)
        return eager(input_ids)

    @torch.no_grad()
    def lightning_prefill(self, input_ids: torch.Tensor):
        """Prefill with the model's configured backend."""
        return self._prefill_eager(input_ids)

    # ------------------------------------------------------------------ decode
    def lightning_step(self, token: torch.Tensor, states: torch.Tensor, pos_tensor: torch.Tensor):
        """One recurrent decode step over all layers; returns (logits, new states)."""
        x = self.drop(self.wte(token) + self.wpe(pos_tensor)[None, :])
        new_states = []
        pending = None
        for index, block in enumerate(self.blocks):
            x, pending, s = block.fused_lightning_step(x, pending, states[index])
            new_states.append(s)
        if ops.decode_head_supported(x, self.ln_f, self.lm_head):
            return ops.decode_head(x, pending, self.ln_f, self.lm_head), torch.stack(new_states, dim=0).contiguous()
        h = self.ln_f(x) if pending is None else self.ln_f.add_forward(x, pending)[1]
        return self.lm_head(h), torch.stack(new_states, dim=0).contiguous()

    def compile_generation(self, *, mode: str = "default", fullgraph: bool = False) -> "ESAModel":
        """torch.compile the fixed-shape decode step (the reference's runtime)."""
        if not hasattr(torch, "compile") or self.device.type != "cuda":
            return self
        key = (mode, bool(fullgraph))
        if self._compiled_lightning_step is not None and self._compiled_lightning_key == key:
            return self
        try:
            self._compiled_lightning_step = torch.compile(self.lightning_step, mode=mode,
                                                          fullgraph=fullgraph, dynamic=False)
            self._compiled_lightning_key = key
        except Exception as exc:
            self._compiled_lightning_step = None
            self._compiled_lightning_key = None
            self._warn_compile_fallback("runtime", exc)
        return self

    def _prefill_for_generate(self, input_ids: torch.Tensor, engine: str, compile_mode: str, use_graph: bool):
        """generate()'s prefill: with graph decoding on a GPU and an eager
        (not compiled) engine, a captured CUDA graph per prompt shape
        (decode_graph.PrefillGraph); otherwise prefill()."""
        spec = parse_engine_spec(engine)
        if use_graph and self.device.type == "cuda" and not spec.compiled and input_ids.ndim == 2:
            ids = input_ids[:, -self.config.block:] if input_ids.size(1) > self.config.block else input_ids
            key = (tuple(ids.shape), spec.backend, spec.compass, self.wte.weight.dtype)
            if key not in self._prefill_graph_failures:
                from .decode_graph import PrefillGraph
                g = self._prefill_graphs.get(key)
                if g is None:
                    g = PrefillGraph(self, tuple(ids.shape), spec.backend, spec.compass)
                    self._prefill_graphs[key] = g
                try:
                    logits, states, T = g.run(ids)
                    return logits.clone(), states, T
                except Exception as exc:  # capture refused (e.g. a host sync on the path)
                    self._prefill_graphs.pop(key, None)
                    self._prefill_graph_failures.add(key)
                    self._warn_compile_fallback("prefill graph", exc)
        return self.prefill(input_ids, engine=engine, compile_mode=compile_mode, fullgraph=False, dynamic=True)

    def _decode_graph(self, batch: int, state_dtype: torch.dtype, temperature, top_k, top_p):
        from .decode_graph import DecodeGraph
        key = (batch, state_dtype, float(temperature), top_k, top_p)
        g = self._decode_graphs.get(key)
        if g is None:
            g = DecodeGraph(self, batch, state_dtype, temperature=temperature, top_k=top_k,
                            top_p=top_p)
            self._decode_graphs[key] = g
        return g

    @torch.inference_mode()
    def generate(self, prompt: str | torch.Tensor | None = None, *, tokenizer: Any | None = None,
                 input_ids: torch.Tensor | None = None, seek: int = 128, prefill: str = "thunder_16",
                 runtime: str = "lightning", temperature: float = 1.0, top_k: int | None = None,
                 top_p: float | None = None, eos_token_id: int | None = None,
                 seed: int | None = None, compile: bool = True, compile_mode: str = "default",
                 progress_interval: int | None = None, stats: bool = False,
                 max_new_tokens: int | None = None, decode_graph: bool = False):
        """Prefill the prompt, then decode `seek` tokens with ESA-Lightning
        (model.py:866-1114).  ``decode_graph=True`` (or runtime
        "lightning_graph") replays a captured CUDA graph per token."""
        if max_new_tokens is not None:
            if seek != 128 and int(seek) != int(max_new_tokens):
                raise ValueError("Pass either seek or max_new_tokens, not conflicting values for both.")
            seek = int(max_new_tokens)
        seek = int(seek)
        if seek <= 0:
            raise ValueError("seek must be positive.")
        if torch.is_tensor(prompt):
            if input_ids is not None:
                raise ValueError("Provide token IDs either positionally or via input_ids, not both.")
            input_ids, prompt = prompt, None
        if input_ids is None:
            if prompt is None or tokenizer is None:
                raise ValueError(
                    "Provide a text prompt with tokenizer, or use the advanced input_ids API.")
            if hasattr(tokenizer, "encode_ordinary"):
                ids = tokenizer.encode_ordinary(prompt)
            elif hasattr(tokenizer, "encode"):
                ids = tokenizer.encode(prompt)
            else:
                raise TypeError("tokenizer must expose encode_ordinary() or encode().")
            input_ids = torch.tensor(ids, dtype=torch.long, device=self.device).unsqueeze(0)
        else:
            input_ids = input_ids.to(self.device)

        rt = str(runtime).strip().lower()
        use_graph = bool(decode_graph) or rt == "lightning_graph"
        if rt == "lightning_graph":
            rt = "lightning"
        runtime_spec = parse_engine_spec(rt)
        if runtime_spec.backend != "lightning":
            raise ValueError("Autoregressive decode currently supports runtime='lightning' only. "
                             "Thunder/Flare/Pulse are selectable prefill engines.")
        compile_runtime = bool(compile or runtime_spec.compiled) and not use_graph

        was_training = self.training
        self.eval()
        try:
            if seed is not None:
                torch.manual_seed(int(seed))
                if self.device.type == "cuda":
                    torch.cuda.manual_seed_all(int(seed))

            def sync() -> None:
                if self.device.type == "cuda":
                    torch.cuda.synchronize(self.device)

            prompt_tokens = int(input_ids.size(1))
            sync()
            total_start = time.perf_counter()
            logits, states, prefill_len = self._prefill_for_generate(input_ids, prefill, compile_mode,
                                                                     use_graph)
            if states.is_cuda:
                states = states.clone()
            sync()
            prefill_seconds = time.perf_counter() - total_start
            next_token = sample_next_token(logits, temperature=temperature, top_k=top_k, top_p=top_p)
            decode_target = seek - 1

            if use_graph and self.device.type == "cuda" and decode_target > 0:
                graph = self._decode_graph(int(input_ids.size(0)), states.dtype, temperature,
                                           top_k, top_p)
                sync()
                decode_start = time.perf_counter()
                generated = graph.run(next_token, states, prefill_len, decode_target,
                                      eos_token_id=eos_token_id)
                states = graph.states
            else:
                generated = [next_token]
                step_fn = self.lightning_step
                using_compiled = False
                if compile_runtime and self.device.type == "cuda":
                    key = (compile_mode, False)
                    if self._compiled_lightning_step is None or self._compiled_lightning_key != key:
                        self.compile_generation(mode=compile_mode, fullgraph=False)
                    if self._compiled_lightning_step is not None:
                        step_fn = self._compiled_lightning_step
                        using_compiled = True
                sync()
                decode_start = time.perf_counter()
                for step in range(decode_target):
                    position = (prefill_len + step) % self.config.block
                    pos_tensor = torch.tensor(position, device=self.device, dtype=torch.long)
                    try:
                        logits, states_out = step_fn(next_token.squeeze(1), states, pos_tensor)
                    except Exception as exc:
                        if not using_compiled:
                            raise
                        self._compiled_lightning_step = None
                        self._compiled_lightning_key = None
                        self._warn_compile_fallback("runtime-execution", exc)
                        step_fn, using_compiled = self.lightning_step, False
                        logits, states_out = step_fn(next_token.squeeze(1), states, pos_tensor)
                    states = states_out.clone() if states_out.is_cuda else states_out
                    next_token = sample_next_token(logits, temperature=temperature, top_k=top_k,
                                                   top_p=top_p)
                    generated.append(next_token)
                    if eos_token_id is not None and bool((next_token == int(eos_token_id)).all()):
                        break
                    if progress_interval and (step + 1) % int(progress_interval) == 0:
                        sync()
                        el = time.perf_counter() - decode_start
                        print(f"ESA-Lightning {step + 1:,}/{decode_target:,} | "
                              f"{(step + 1) / max(el, 1e-9):,.2f} tok/s")
                generated = torch.cat(generated, dim=1)
            sync()
            decode_seconds = time.perf_counter() - decode_start if decode_target > 0 else 0.0
            total_seconds = time.perf_counter() - total_start
            generated_ids = generated if torch.is_tensor(generated) else torch.cat(generated, dim=1)
            sequences = torch.cat([input_ids, generated_ids], dim=1)
            state_bytes = int(states.numel() * states.element_size())
            n_gen = int(generated_ids.size(1))
            st = GenerationStats(
                prompt_tokens=prompt_tokens, prefill_tokens=int(prefill_len),
                generated_tokens=n_gen, decode_steps=max(0, n_gen - 1),
                prefill_seconds=prefill_seconds, decode_seconds=decode_seconds,
                decode_tok_s=max(0, n_gen - 1) / max(decode_seconds, 1e-9),
                total_seconds=total_seconds, state_bytes=state_bytes,
                state_mb=state_bytes / 1024 ** 2)
            result = GenerationResult(sequences=sequences, generated_ids=generated_ids, stats=st)
            if tokenizer is not None:
                if sequences.size(0) == 1:
                    result.text = tokenizer.decode(sequences[0].detach().cpu().tolist())
                else:
                    result.text = [tokenizer.decode(r.detach().cpu().tolist()) for r in sequences]
            if stats:
                return result
            if result.text is not None:
                return result.text
            return sequences
        finally:
            self.train(was_training)

    @torch.inference_mode()
    def generate_ids(self, input_ids: torch.Tensor, *, seek: int = 128, **kwargs: Any):
        """Token-level generation API."""
        return self.generate(input_ids=input_ids, seek=seek, **kwargs)

    def model_info(self) -> dict[str, Any]:
        return {**asdict(self.config), "parameters": sum(p.numel() for p in self.parameters()),
                "device": str(self.device), "generation_engine": "ESA-Lightning"}

    # ------------------------------------------------------------------ persistence
    def save(self, path: str | Path, *, metadata: dict[str, Any] | None = None) -> Path:
        """Write config.json, model.pt (state_dict) and metadata.json (model.py:1154-1215)."""
        path = Path(path)
        path.mkdir(parents=True, exist_ok=True)
        (path / "config.json").write_text(json.dumps(asdict(self.config), indent=2), encoding="utf-8")
        torch.save(self.state_dict(), path / "model.pt")
        meta = {"format_version": self.config.format_version, "architecture": "ESAModel",
                "generation_engine": "ESA-Lightning", "backend": self.config.backend}
        if metadata:
            meta.update(metadata)
        (path / "metadata.json").write_text(json.dumps(meta, indent=2, default=str), encoding="utf-8")
        return path

    @classmethod
    def load(cls, path: str | Path, *, device: str | torch.device = "cpu", strict: bool = True):
        """Rebuild from config.json and load model.pt (model.py:1217-1256)."""
        path = Path(path)
        config = ESAModelConfig.from_dict(json.loads((path / "config.json").read_text(encoding="utf-8")))
        model = cls(config, device=str(device))
        state = torch.load(path / "model.pt", map_location=device, weights_only=True)
        model.load_state_dict(state, strict=strict)
        return model.to(device)
