"""PredictorState: the per-request controller of the SQ3.25 recurrent state.

Same constructor and methods as scripts/fp4_zero_predictor_codec_v1.py:239-367
(inheriting mamba2_recall/state_quant.py:41-370): install/close (context manager),
reset(batch_size), backbone(ids, reset=False) -> fp16 hidden after norm_f,
storage_descriptor(), assert_finite_cache(), cache_breakdown().  Instead of
monkey-patching mamba_ssm mixers, one native call (sq_model_forward in libsq325.so)
runs every layer.  The controller owns the request caches (six PackedState tensors per
layer plus a conv ring) and latches `_failed` on any error until the next reset.
"""
from __future__ import annotations

import ctypes as C
import weakref

import torch

from . import _lib
from .codec import allocate_state, layout_descriptor, layout_index, validate_state
from .model import D_MODEL, D_XBC

_OWNERS = weakref.WeakKeyDictionary()


class _LayerCache:
    def __init__(self, conv, state):
        self.conv = conv          # fp16 ring [batch, 4, 10240], slot = position % 4
        self.state = state        # PackedState
        self.tokens = 0


class PredictorState:
    def __init__(self, model, table, layouts, bases, scales, predictors):
        n = model.n_layer
        self.model = model
        self.device = model.device
        if not isinstance(table, torch.Tensor) or table.dtype != torch.uint8 or tuple(table.shape) != (n, 8, 128):
            raise ValueError(f'Expected permutations of shape [{n},8,128]')
        cpu = table.detach().cpu().contiguous()
        if not torch.equal(cpu.sort(dim=-1).values, torch.arange(128, dtype=torch.uint8).expand_as(cpu)):
            raise ValueError('Every state group must be a permutation of 0..127')
        self.permutations = cpu.to(self.device).contiguous()
        if not isinstance(layouts, (tuple, list)) or len(layouts) != n:
            raise ValueError(f'Exactly {n} per-layer layout names are required')
        self.layouts = tuple(layouts)
        for layout in self.layouts:
            layout_descriptor(layout)
        if len(bases) != n or len(scales) != n or len(predictors) != n:
            raise ValueError(f'Exactly {n} static bases/scales/predictors required')
        self.bases, self.latent_scales, self.predictors = [], [], []
        for layer, layout in enumerate(self.layouts):
            spec = layout_descriptor(layout)
            basis = bases[layer].to(device=self.device, dtype=torch.float16).contiguous()
            scale = scales[layer].to(device=self.device, dtype=torch.float16).contiguous()
            pred = predictors[layer].to(device=self.device, dtype=torch.float16).contiguous()
            if (tuple(basis.shape) != (8, spec['nzero'], 2) or tuple(scale.shape) != (8, 2) or
                    tuple(pred.shape) != (8, spec['n8'] + spec['n4'] + 2, spec['nzero']) or
                    not bool(torch.isfinite(basis).all()) or not bool(torch.isfinite(scale).all()) or
                    not bool(torch.isfinite(pred).all()) or not bool((scale > 0).all())):
                raise ValueError('Static predictor/basis/scale allocation differs')
            self.bases.append(basis); self.latent_scales.append(scale); self.predictors.append(pred)
        self._handle = None
        self._cache = []
        self._batch_size = None
        self._failed = False
        self._installed = False
        self._inside_backbone = False
        self._reserved = 0
        self._exact_projections = False

    # ------------------------------------------------------------------ lifecycle
    def install(self):
        if self._installed:
            raise RuntimeError('Controller is already installed')
        owner = _OWNERS.get(self.model)
        if owner is not None and owner() is not None:
            raise RuntimeError('Another controller owns this model')
        _OWNERS[self.model] = weakref.ref(self)
        try:
            h = C.c_void_p()
            cfg = _lib.ModelConfig(self.model.n_layer, self.model.vocab, self.model.eps)
            _lib.call('sq_model_create', C.byref(cfg), C.byref(h))
            self._handle = h
            _lib.call('sq_model_set_exact_skinny', h, int(self._exact_projections))
            for i, (L, layout) in enumerate(zip(self.model.layers, self.layouts)):
                d = _lib.LayerDesc()
                d.in_proj, d.out_proj = L.in_proj.cabi(), L.out_proj.cabi()
                d.norm_weight, d.conv_weight, d.conv_bias = (L.norm_weight.data_ptr(), L.conv_weight.data_ptr(),
                                                             L.conv_bias.data_ptr())
                d.A, d.D, d.dt_bias, d.gated_norm_weight = (L.A.data_ptr(), L.D.data_ptr(), L.dt_bias.data_ptr(),
                                                            L.gated_norm_weight.data_ptr())
                d.layout = layout_index(layout)
                d.permutation = self.permutations[i].data_ptr()
                d.basis, d.latent_scale, d.predictor = (self.bases[i].data_ptr(), self.latent_scales[i].data_ptr(),
                                                        self.predictors[i].data_ptr())
                _lib.call('sq_model_set_layer', h, i, C.byref(d))
            e, hd = self.model.embedding.cabi(), self.model.lm_head.cabi()
            _lib.call('sq_model_set_globals', h, C.byref(e), C.byref(hd), _lib.ptr(self.model.norm_f))
            self._sync_adapter()
            self._installed = True
        except Exception:
            self.close()
            raise
        return self

    def time_projection_gemm(self, enable=True):
        """Measurement hook: bracket every later large-M in_proj tcgen05 GEMM launch (prompts,
        scoring windows) with a pair of CUDA events on its stream (sq_model_time_gemm)."""
        if self._handle is None:
            raise RuntimeError('install() the model first')
        _lib.call('sq_model_time_gemm', self._handle, int(bool(enable)))

    def projection_gemm_time(self):
        """(device seconds, launches) of the GEMM launches recorded since
        time_projection_gemm; the records are then discarded."""
        sec, n = C.c_double(), C.c_int64()
        _lib.call('sq_model_gemm_time', self._handle, C.byref(sec), C.byref(n))
        return sec.value, n.value

    def set_exact_projections(self, exact=True):
        """One-token decode steps and the greedy head use the factored global scale by
        default (fp16 products E2M1*E4M3 on the tensor cores, fp32 global scale once per
        output).  exact=True rounds every weight to fp16 first, the reference's decoded-weight
        numerics, at about three ALU instructions per weight.  Prompts and scoring always use
        the exactly decoded weights."""
        self._exact_projections = bool(exact)
        if self._handle is not None:
            _lib.call('sq_model_set_exact_skinny', self._handle, int(self._exact_projections))
        return self

    def _sync_adapter(self):
        bank = getattr(self.model, 'adapter', None)
        for i in range(self.model.n_layer):
            if bank is None:
                _lib.call('sq_model_set_adapter', self._handle, i, None, None, None, None, 0)
            else:
                _lib.call('sq_model_set_adapter', self._handle, i, _lib.ptr(bank.V[i]), _lib.ptr(bank.g[i]),
                          _lib.ptr(bank.w[i]), _lib.ptr(bank.b[i]), int(bank.gate_mode == 'hard'))

    def __enter__(self):
        return self.install()

    def __exit__(self, *exc):
        self.close()
        return False

    def close(self):
        if self._handle is not None:
            torch.cuda.synchronize(self.device)
            _lib.load().sq_model_destroy(self._handle)
            self._handle = None
        self._installed = False
        owner = _OWNERS.get(self.model)
        if owner is not None and owner() is self:
            del _OWNERS[self.model]
        self.clear()

    def clear(self):
        self._cache = []
        self._batch_size = None
        self._failed = False

    @torch.no_grad()
    def reset(self, batch_size=1):
        if not self._installed or type(batch_size) is not int or batch_size <= 0:
            raise ValueError('Installed controller and positive batch required')
        self.clear()
        for i, layout in enumerate(self.layouts):
            conv = torch.zeros(batch_size, 4, D_XBC, device=self.device, dtype=torch.float16)
            state = allocate_state(batch_size, 128, 64, 128, self.device, layout=layout)
            validate_state(state, self.device, layout)
            t = state.tensors
            _lib.call('sq_model_bind_state', self._handle, i, batch_size, *(_lib.ptr(t[k]) for k in
                      ('lo', 'hi', 'q4', 'latent', 's8', 's4')), _lib.ptr(conv))
            self._cache.append(_LayerCache(conv, state))
        self._batch_size = batch_size
        # 56 layers: batch * (28,499,968 - 57,344) + 57,344 (fp4_zero_predictor_codec_v1.py:277-279)
        per_layer = 4 * D_XBC * 2 + 128 * 64 * 52
        n = self.model.n_layer
        expected = batch_size * n * per_layer + n * 8 * 128
        if self.cache_breakdown()['total_bytes'] != expected:
            raise RuntimeError('Latent request cache violates fixed physical budget')
        return self

    def reserve(self, max_tokens):
        if max_tokens > self._reserved:
            _lib.call('sq_model_reserve', self._handle, int(max_tokens))
            self._reserved = int(max_tokens)

    # ------------------------------------------------------------------ execution
    @torch.no_grad()
    def backbone(self, ids, reset=False, out=None):
        """Hidden states fp16 [batch, tokens, 4096] after norm_f, advancing the caches."""
        if not self._installed:
            raise RuntimeError('Controller is not installed')
        if not isinstance(ids, torch.Tensor) or ids.ndim != 2 or ids.shape[1] == 0:
            raise ValueError('Input IDs must be nonempty [batch,tokens]')
        if ids.device != self.device or ids.dtype != torch.long:
            raise ValueError('Input IDs must be CUDA int64 on the model device')
        if self._inside_backbone:
            raise RuntimeError('Concurrent/reentrant backbone invocation is unsupported')
        if reset or not self._cache:
            self.reset(ids.shape[0])
        if self._failed:
            raise RuntimeError('Controller is inactive or failed; reset before reusing it')
        if ids.shape[0] != self._batch_size:
            raise RuntimeError('Batch shape changed without a reset')
        if len({e.tokens for e in self._cache}) != 1:
            raise RuntimeError('Per-layer cache positions disagree; reset the request')
        B, T = ids.shape
        ids = ids.contiguous()
        self.reserve(B * T)
        if out is None:
            out = torch.empty((B, T, D_MODEL), device=self.device, dtype=torch.float16)
        self._inside_backbone = True
        try:
            _lib.call('sq_model_forward', self._handle, _lib.ptr(ids), B, T, self._cache[0].tokens, _lib.ptr(out),
                      _lib.stream_ptr())
            for e in self._cache:
                e.tokens += T
            return out
        except Exception:
            self._failed = True
            raise
        finally:
            self._inside_backbone = False

    @torch.no_grad()
    def mixer_forward(self, layer, u, out=None):
        """One mixer layer (the reference's patched `mixer.forward`, PredictorState._forward
        fp4_zero_predictor_codec_v1.py:314-367): u fp16 [batch, tokens, 4096] is the Block's
        normed input; returns the mixer output and advances this layer's cache position."""
        if not self._installed:
            raise RuntimeError('Controller is not installed')
        if not self._cache:
            raise RuntimeError('reset() the controller before running a layer')
        if self._failed:
            raise RuntimeError('Controller is inactive or failed; reset before reusing it')
        if u.ndim != 3 or u.shape[0] != self._batch_size or u.shape[2] != D_MODEL or u.dtype != torch.float16 \
                or u.device != self.device:
            raise ValueError('u must be CUDA fp16 [batch, tokens, 4096] matching the reset batch')
        B, T = u.shape[:2]
        u = u.contiguous()
        self.reserve(B * T)
        out = out if out is not None else torch.empty_like(u)
        e = self._cache[layer]
        try:
            _lib.call('sq_model_mixer_forward', self._handle, layer, _lib.ptr(u), B, T, e.tokens, _lib.ptr(out),
                      _lib.stream_ptr())
        except Exception:
            self._failed = True
            raise
        e.tokens += T
        return out

    @torch.no_grad()
    def score(self, hidden, targets, out=None):
        """Per-row next-token NLL (fp32) of fp16 logits lm_head(hidden).float()."""
        h2 = hidden.reshape(-1, D_MODEL).contiguous()
        t = targets.reshape(-1).to(device=self.device, dtype=torch.long).contiguous()
        if t.numel() != h2.shape[0]:
            raise ValueError('One target per hidden row required')
        self.reserve(h2.shape[0])
        nll = out if out is not None else torch.empty(h2.shape[0], device=self.device, dtype=torch.float32)
        _lib.call('sq_model_score', self._handle, _lib.ptr(h2), h2.shape[0], _lib.ptr(t), _lib.ptr(nll),
                  _lib.stream_ptr())
        return nll

    @torch.no_grad()
    def greedy(self, hidden, logits=None, tokens=None):
        h2 = hidden.reshape(-1, D_MODEL).contiguous()
        rows = h2.shape[0]
        self.reserve(max(rows, 1))
        tok = tokens if tokens is not None else torch.empty(rows, device=self.device, dtype=torch.long)
        _lib.call('sq_model_greedy', self._handle, _lib.ptr(h2), rows, _lib.ptr(logits), _lib.ptr(tok),
                  _lib.stream_ptr())
        return tok

    # ------------------------------------------------------------------ graphed decode
    @torch.no_grad()
    def capture_decode(self, tokens):
        """Capture the one-token greedy step (forward + lm_head + argmax) as CUDA graphs.

        `tokens` is an int64 [batch] device tensor that the graph reads as this step's input
        and overwrites with the argmax token, so replays chain without host round trips.
        The conv ring slot depends on position % 4, so four graphs are captured (one per
        residue) and replayed in turn.  Requires a prefilled request (tokens > 0)."""
        if not self._cache or self._cache[0].tokens == 0:
            raise RuntimeError('Prefill the request before capturing decode graphs')
        B = self._batch_size
        if tokens.shape != (B,) or tokens.dtype != torch.long or tokens.device != self.device:
            raise ValueError('tokens must be CUDA int64 [batch]')
        self.reserve(B)
        self._graph_tokens = tokens
        self._graph_hidden = torch.empty((B, 1, D_MODEL), device=self.device, dtype=torch.float16)
        side = torch.cuda.Stream(self.device)
        side.wait_stream(torch.cuda.current_stream(self.device))
        self._graphs = []
        with torch.cuda.stream(side):
            for r in range(4):
                g = torch.cuda.CUDAGraph()
                with torch.cuda.graph(g, stream=side):
                    sp = C.c_void_p(side.cuda_stream)
                    _lib.call('sq_model_forward', self._handle, _lib.ptr(tokens), B, 1, 4 + r,
                              _lib.ptr(self._graph_hidden), sp)
                    _lib.call('sq_model_greedy', self._handle, _lib.ptr(self._graph_hidden), B, None,
                              _lib.ptr(tokens), sp)
                self._graphs.append(g)
        torch.cuda.current_stream(self.device).wait_stream(side)
        return self._graphs

    @torch.no_grad()
    def replay_decode(self, steps):
        """Advance `steps` greedy tokens by graph replay; returns int64 [steps, batch]."""
        out = torch.empty((steps, self._batch_size), device=self.device, dtype=torch.long)
        for i in range(steps):
            self._graphs[self._cache[0].tokens % 4].replay()
            for e in self._cache:
                e.tokens += 1
            out[i].copy_(self._graph_tokens)
        return out

    @torch.no_grad()
    def decode_persistent(self, tokens, steps):
        """Greedy decode at batch 1 with one persistent cooperative kernel launch for all
        `steps` tokens (every layer, the final norm, lm_head and argmax per token).  `tokens` is an int64 [1]
        device tensor holding the token to feed first; it is overwritten with every pick.
        Returns int64 [steps, 1] picks.  Same tokens and states as `replay_decode`, with the
        projection numerics that set_exact_projections selects (factored scale by default)."""
        if not self._cache or self._cache[0].tokens == 0:
            raise RuntimeError('Prefill the request before decoding')
        if self._batch_size != 1:
            raise ValueError('The persistent decode kernel runs batch 1')
        if tokens.shape != (1,) or tokens.dtype != torch.long or tokens.device != self.device:
            raise ValueError('tokens must be CUDA int64 [1]')
        if steps <= 0:
            raise ValueError('steps must be positive')
        self.reserve(1)
        out = torch.empty((steps, 1), device=self.device, dtype=torch.long)
        with torch.cuda.device(self.device):
            _lib.call('sq_model_decode', self._handle, _lib.ptr(tokens), self._cache[0].tokens, steps,
                      _lib.ptr(out), _lib.stream_ptr())
        for e in self._cache:
            e.tokens += steps
        return out

    def capture_layers(self, rows):
        """Record every layer's mixer output during later backbone calls of at most `rows`
        tokens (batch * tokens): returns the fp16 [n_layer, rows, 4096] buffer that each
        forward fills.  capture_layers(0) turns it off."""
        if not self._installed:
            raise RuntimeError('Controller is not installed')
        if rows <= 0:
            _lib.call('sq_model_set_capture', self._handle, None, 0)
            self._capture = None
            return None
        self._capture = torch.empty((self.model.n_layer, rows, D_MODEL), device=self.device, dtype=torch.float16)
        _lib.call('sq_model_set_capture', self._handle, _lib.ptr(self._capture), rows)
        return self._capture

    def check(self):
        """Synchronise and raise if a device-side check failed (bad token id, expired wait)."""
        _lib.call('sq_model_check', self._handle, _lib.stream_ptr())

    # ------------------------------------------------------------------ inspection
    def conv_chronological(self, layer):
        """The conv cache in the reference's [batch, 10240, 4] order (slot 3 = newest)."""
        e = self._cache[layer]
        pos = e.tokens
        idx = [(pos - 4 + k) % 4 for k in range(4)]
        return e.conv[:, idx, :].transpose(1, 2).contiguous()

    def cache_breakdown(self):
        conv = sum(e.conv.numel() * e.conv.element_size() for e in self._cache)
        state = sum(int(e.state.nbytes) for e in self._cache)
        scales = sum(t.numel() * t.element_size() for e in self._cache for k, t in e.state.tensors.items()
                     if k in ('s4', 's8'))
        tables = self.permutations.numel() * self.permutations.element_size()
        return {'mode': 'sq3p25_latent', 'batch_size': self._batch_size, 'allocated_layers': len(self._cache),
                'conv_fp16_bytes': conv, 'ssm_payload_bytes': state - scales, 'ssm_scale_bytes': scales,
                'ssm_total_bytes': state, 'permutation_bytes': tables, 'total_bytes': conv + state + tables,
                'tokens_per_layer': [e.tokens for e in self._cache]}

    def storage_descriptor(self):
        layers = []
        for layer, (e, layout, basis, scale, pred) in enumerate(zip(self._cache, self.layouts, self.bases,
                                                                     self.latent_scales, self.predictors)):
            validate_state(e.state, self.device, layout)
            layers.append(dict(**layout_descriptor(layout), layer=layer, state_shape=list(e.state.shape),
                               state_bytes=e.state.nbytes,
                               tensors={k: dict(shape=list(v.shape), dtype=str(v.dtype),
                                                storage_bytes=v.untyped_storage().nbytes())
                                        for k, v in e.state.tensors.items()},
                               conv_shape=list(e.conv.shape), conv_storage_bytes=e.conv.untyped_storage().nbytes(),
                               static_basis_bytes=basis.untyped_storage().nbytes(),
                               static_scale_bytes=scale.untyped_storage().nbytes(),
                               static_predictor_bytes=pred.untyped_storage().nbytes()))
        return dict(format='FP4_LATENT_STATE_STORAGE_V1', layouts=list(self.layouts), row_bytes=52, payload_bytes=48,
                    scale_bytes=4, permutation_storage_bytes=self.permutations.untyped_storage().nbytes(),
                    total_cache_bytes=self.cache_breakdown()['total_bytes'],
                    static_basis_bytes=sum(x.untyped_storage().nbytes() for x in self.bases),
                    static_scale_bytes=sum(x.untyped_storage().nbytes() for x in self.latent_scales),
                    static_predictor_bytes=sum(x.untyped_storage().nbytes() for x in self.predictors), layers=layers)

    def assert_finite_cache(self):
        values = [e.conv for e in self._cache]
        values.extend(t for e in self._cache for t in e.state.tensors.values() if t.is_floating_point())
        if values and not all(bool(torch.isfinite(v.float()).all()) for v in values):
            raise FloatingPointError('Nonfinite persistent latent/scale/convolution cache')
        return True
