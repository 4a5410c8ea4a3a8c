"""B200Engine: the BaseEngine implementation that owns the decoder forward.

load() builds one model replica (tensor-parallel over ``tp_size`` ranks, one
process per GPU), sizes the paged KV cache from free device memory, and starts
the scheduler loop thread on rank 0. generate_streaming() keeps the
reference's contract (core/engine_transformers.py:1204-1518): chat template ->
token stream through ``on_token`` -> cleaned answer, and the same
``_last_gen_stats`` keys (tokens, prompt_tokens, completion_tokens,
finish_reason, wall_time, tok_per_sec, ttft, decode_tok_per_sec).
generate() is the batch API: many token-id prompts in, completions out.
"""

from __future__ import annotations

import logging
import os
import queue
import threading
import time

import torch

from b200serve.core.config import EngineConfig
from b200serve.core.engine_base import BaseEngine
from b200serve.core.inference import _clean_response, strip_think_blocks, STOP_STRINGS
from b200serve.engine.kv_cache import BLOCK, KVCache
from b200serve.engine.sampler import SamplingParams
from b200serve.engine.scheduler import Request, Scheduler
from b200serve.engine.tokenizer import IncrementalDecoder, load_tokenizer

_log = logging.getLogger(__name__)


def _dtype(name):
    return {"bfloat16": torch.bfloat16, "bf16": torch.bfloat16, "float32": torch.float32,
            "fp32": torch.float32}[name]


def _safetensors_getter(path):
    """name -> tensor (or None) over the safetensors files of a checkpoint directory."""
    import glob
    from safetensors import safe_open
    where = {}
    for f in sorted(glob.glob(os.path.join(path, "*.safetensors"))):
        h = safe_open(f, framework="pt")
        for k in h.keys():
            where[k] = h
    return lambda name: where[name].get_tensor(name) if name in where else None


def _window_pages(max_batch: int, window_tokens: int) -> int:
    """Pages of the bf16 residual-window pool: a ring of window / 16 + 1 pages per sequence slot,
    one more slot for the padded rows of a decode bucket."""
    return (max_batch + 1) * (window_tokens // BLOCK + 1)


def _kv_layers(mc) -> int:
    return sum(1 for i in range(mc.num_layers) if mc.has_kv(i))


class B200Engine(BaseEngine):
    stream_starts_in_think = True

    def __init__(self, config: EngineConfig = None, weights=None, tokenizer=None, model_config=None, mtp=None):
        self.config = (config or EngineConfig()).validate()
        self._injected_model_cfg = model_config
        self._injected_weights = weights
        self._injected_mtp = mtp                  # models.mtp.MTPWeights for spec_mtp
        self._injected_tokenizer = tokenizer
        self.model_cfg = None
        self.weights = None
        self.kv = None
        self.runner = None
        self.scheduler = None
        self.tokenizer = None
        self.comm = None
        self._loaded_model = None
        self._thread = None
        self._stop = threading.Event()
        self._wake = threading.Condition()
        self._error = None
        self._stats_tls = threading.local()
        self._shared_stats = None
        self.rank = 0
        self.world = 1
        self._step_t0 = None        # start of the step in progress (watchdog)
        self.stalled = False
        self._watch = None

    # ------------------------------------------------------------ per-request stats
    @property
    def _last_gen_stats(self):
        """Stats of the last generate_streaming call made by THIS thread (the reference's
        attribute name and keys). Concurrent requests each run in their own thread, so one
        request never reads another's usage or finish_reason; a thread that has not generated
        sees the most recent call of any thread."""
        mine = getattr(self._stats_tls, "stats", None)
        return mine if mine is not None else self._shared_stats

    @_last_gen_stats.setter
    def _last_gen_stats(self, value):
        self._stats_tls.stats = value
        self._shared_stats = value

    # ------------------------------------------------------------ lifecycle
    def is_loaded(self) -> bool:
        return self.runner is not None

    def needs_reload(self) -> bool:
        from b200serve.core.config import get_active_model_name
        return self._loaded_model is not None and self._loaded_model != self.config.model

    def load(self, status_callback=None):
        if self.is_loaded():
            return
        cfgE = self.config
        say = status_callback or (lambda m: _log.info(m))
        from b200serve.models.config import get_model_config
        from b200serve.parallel import dist as pdist
        self.rank, self.world = pdist.rank_world()
        tp = cfgE.tp_size
        if tp > 1 and self.world != tp:
            raise RuntimeError(f"tp_size={tp} needs {tp} ranks (torchrun), found world={self.world}")
        if cfgE.device == "cuda" and torch.cuda.is_available():
            dev = torch.device("cuda", pdist.local_rank() if tp > 1 else torch.cuda.current_device())
            torch.cuda.set_device(dev)
        else:
            dev = torch.device("cpu")
        self.device = dev
        if self._injected_model_cfg is None and not os.path.exists(cfgE.model):
            # a registered model (core/model_inventory.py): its checkpoint path and serving fields
            from b200serve.core.model_inventory import engine_overrides
            try:
                ov = engine_overrides(cfgE.model)
            except (OSError, ValueError):
                ov = None
            if ov:
                for k, v in ov.items():
                    if k != "tp_size":            # the launch decides the ranks
                        setattr(cfgE, k, v)
        mc = self._injected_model_cfg or get_model_config(cfgE.model, cfgE.num_layers_override)
        self.model_cfg = mc
        if cfgE.max_seq <= 0:
            self._plan_max_seq(mc, dev)
        dtype = _dtype(cfgE.dtype)
        say(f"b200: building {mc.name} ({mc.num_params() / 1e9:.2f}B params) tp={tp} on {dev}")
        self.weights = self._injected_weights or self._load_weights(mc, dtype, dev)
        if cfgE.quantize:
            if cfgE.quantize != "q4_k_m" or dev.type != "cuda":
                raise ValueError("quantize='q4_k_m' needs a CUDA device")
            if mc.is_moe or mc.is_hybrid or mc.attn_output_gate:
                raise NotImplementedError("load-time 4-bit quantisation covers dense attention models")
            if (mc.intermediate_size // cfgE.tp_size) % 64 or mc.hidden_size % 256:
                raise NotImplementedError("4-bit blocks need hidden % 256 == 0 and FFN width % 64 == 0")
            from b200serve.models.gguf_gpu import quantize_model_q4_k_m
            say("b200: quantising projections to Q4_K_M blocks")
            quantize_model_q4_k_m(self.weights, mc)
        self.comm = pdist.make_comm(cfgE, dev, self.model_cfg) if tp > 1 else None
        nkv_local = max(1, mc.num_kv_heads // tp)
        num_blocks = self._size_kv(mc, nkv_local, dtype, dev)
        # hybrid models page K/V for their full-attention layers only
        self.kv = KVCache(_kv_layers(mc), num_blocks, nkv_local, mc.head_dim, dtype=dtype, device=dev,
                          kv_format=cfgE.kv_format, key_bits=cfgE.kv_key_bits, value_bits=cfgE.kv_value_bits)
        kv_b, nb = None, 0
        if cfgE.kv_format == "turboquant" and cfgE.kv_boundary_layers > 0:
            nb = cfgE.kv_boundary_layers
            n_kv = _kv_layers(mc)
            kv_b = KVCache(min(n_kv, 2 * nb), num_blocks, nkv_local, mc.head_dim, dtype=dtype, device=dev)
        kv_w, rw = None, 0
        if cfgE.kv_format == "turboquant" and cfgE.kv_residual_tokens > 0:
            rw = (cfgE.kv_residual_tokens + BLOCK - 1) // BLOCK * BLOCK
            kv_w = KVCache(_kv_layers(mc), _window_pages(cfgE.max_batch, rw), nkv_local, mc.head_dim, dtype=dtype,
                           device=dev)
        from b200serve.engine.runner import ModelRunner
        runner = ModelRunner(mc, self.weights, self.kv, comm=self.comm, device=dev, max_batch=cfgE.max_batch,
                             kv_boundary=kv_b, boundary_layers=nb, kv_window=kv_w, window_tokens=rw,
                             max_seq=cfgE.max_seq, use_graphs=cfgE.cuda_graphs)
        if tp > 1:
            from b200serve.parallel.worker import BroadcastRunner
            runner = BroadcastRunner(runner, self.comm)
        self.runner = runner
        if cfgE.spec_mtp:
            self._attach_mtp(mc, dtype, dev)
        self._attach_vision(mc, dtype, dev)
        # a prefix-cache hit would skip tokens whose recurrent state a hybrid model needs
        self.scheduler = Scheduler(runner, num_blocks, max_batch=cfgE.max_batch, prefill_chunk=cfgE.prefill_chunk,
                                   max_seq=cfgE.max_seq, prefix_cache=not mc.is_hybrid and kv_w is None,
                                   spec_ngram=0 if mc.is_hybrid else cfgE.spec_ngram,
                                   spec_mtp=cfgE.spec_mtp and getattr(runner, "mtp", None) is not None)
        self.tokenizer = self._injected_tokenizer or load_tokenizer(self._model_path(), mc.vocab_size)
        vl = getattr(self.runner, "vl", None)
        if vl is not None and hasattr(self.tokenizer, "add_special"):
            # a checkpoint without tokenizer files: the image markers still encode to their ids
            t = vl.tokens
            self.tokenizer.add_special({"<|vision_start|>": t.vision_start, "<|image_pad|>": t.image,
                                        "<|vision_end|>": t.vision_end})
        from b200serve.core import inference
        inference._tokenizer = self.tokenizer
        self._loaded_model = cfgE.model
        say(f"b200: ready, {num_blocks} KV pages ({num_blocks * BLOCK} tokens)")

    def _attach_vision(self, mc, dtype, dev):
        """The vision tower of a vision-language checkpoint (``vision_config`` and ``model.visual.*``
        tensors), bound to the runner. Single-rank engines."""
        path = self.config.model
        cfg_path = os.path.join(path, "config.json") if os.path.isdir(path) else ""
        if not cfg_path or not os.path.exists(cfg_path) or self.config.weights != "safetensors":
            return
        import json
        with open(cfg_path) as fh:
            hf = json.load(fh)
        if "vision_config" not in hf:
            return
        if self.config.tp_size > 1:
            _log.warning("b200: the vision tower runs on single-rank engines; images are refused")
            return
        from b200serve.models.qwen_vl import VisionLanguage
        vl = VisionLanguage.from_checkpoint(hf, _safetensors_getter(path), mc, dev, dtype)
        if vl is not None:
            self.runner.vl = vl

    def prepare_images(self, prompt_ids, images):
        """(expanded prompt ids, multimodal input) for a prompt with image placeholders."""
        vl = getattr(self.runner, "vl", None)
        if vl is None:
            raise ValueError("this model has no vision tower; images are not accepted")
        return vl.prepare(list(prompt_ids), images)

    def generate_images(self, prompt_ids, images, params: SamplingParams = None, timeout: float = None):
        """One prompt (token ids with image placeholders) with PIL images -> finished Request."""
        self.load()
        params = params or SamplingParams()
        ids, mm = self.prepare_images(prompt_ids, images)
        stop_ids = set() if params.ignore_eos else self.tokenizer.stop_ids
        req = Request(prompt=ids, params=params, stop_ids=stop_ids)
        req.mm = mm
        self.submit(req)
        if not req.done_event.wait(timeout):
            raise TimeoutError(f"{req.rid} did not finish")
        return req

    def _attach_mtp(self, mc, dtype, dev):
        """Bind the MTP head (checkpoint ``mtp.*`` tensors, or a random head for random weights)
        to the runner. Single rank, attention-only trunks: a hybrid trunk's recurrent state
        cannot be rolled back past a rejected draft."""
        from b200serve.models import mtp as MTP
        cfgE = self.config
        if cfgE.tp_size > 1 or mc.is_hybrid or mc.is_moe:
            _log.warning("b200: MTP drafting runs on one rank with an attention-only dense trunk; off")
            return
        head = self._injected_mtp
        if head is None and cfgE.weights == "random":
            head = MTP.random_mtp(mc, seed=cfgE.seed, std=cfgE.init_std, dtype=dtype, device=dev)
        elif head is None and cfgE.weights == "safetensors":
            head = MTP.mtp_from_getter(mc, _safetensors_getter(cfgE.model), dtype=dtype, device=dev)
        if head is None:
            _log.warning("b200: spec_mtp set but the checkpoint has no MTP head; off")
            return
        self.runner.mtp = MTP.MTPHead(mc, self.runner.decoder, head, dev)

    def _plan_max_seq(self, mc, dev):
        """max_seq = 0: the longest context tier whose KV fits next to the weights."""
        from b200serve.core.ctx_planner import plan_context
        cfgE = self.config
        if dev.type == "cuda":
            free, _ = torch.cuda.mem_get_info(dev)
            free -= int(mc.num_params() * 2 / cfgE.tp_size)       # bf16 weights still to load
        else:
            free = 16 << 30
        state = 0
        if mc.is_hybrid:
            from b200serve.models.hybrid import LinearState
            state = LinearState.bytes_per_slot(mc, cfgE.tp_size)
        ctx = plan_context(mc, free, cfgE.max_batch, cfgE.tp_size, cfgE.kv_format, state_bytes_per_seq=state)
        if ctx == 0:
            raise RuntimeError("not even a 4096-token context fits; lower max_batch or use a smaller KV format")
        cfgE.max_seq = ctx
        _log.info(f"b200: planned context {ctx} tokens for {cfgE.max_batch} sequences")

    def _model_path(self):
        m = self.config.model
        return m if os.path.exists(m) else None

    def _load_weights(self, mc, dtype, dev):
        cfgE = self.config
        if not cfgE.shard_cache:
            return self._load_weights_uncached(mc, dtype, dev)
        import torch.distributed as dist
        from b200serve.models import shard_cache as SC
        source = cfgE.model if cfgE.weights != "random" else f"random:{cfgE.seed}:{cfgE.init_std}"
        fp = SC.fingerprint(mc, source)
        tp = cfgE.tp_size
        rank = self.rank if tp > 1 else 0
        if SC.valid(cfgE.shard_cache, fp, tp, dtype):
            _log.info(f"b200: weights from the shard cache {cfgE.shard_cache}")
            return SC.load(cfgE.shard_cache, rank, tp, device=dev)
        w = self._load_weights_uncached(mc, dtype, dev)
        barrier = dist.barrier if (tp > 1 and dist.is_initialized()) else None
        try:
            SC.save(w, cfgE.shard_cache, fp, dtype, barrier=barrier)
        except TypeError as e:     # block-quantised layers stay uncached
            _log.warning(f"b200: shard cache not written: {e}")
        return w

    def _load_weights_uncached(self, mc, dtype, dev):
        cfgE = self.config
        from b200serve.models import weights as W
        kw = dict(tp_rank=self.rank if cfgE.tp_size > 1 else 0, tp_size=cfgE.tp_size,
                  ep_rank=self.rank if cfgE.ep_size > 1 else 0, ep_size=cfgE.ep_size, dtype=dtype, device=dev)
        if cfgE.weights == "random":
            return W.random_weights(mc, seed=cfgE.seed, std=cfgE.init_std, **kw)
        if cfgE.weights == "safetensors":
            return W.load_safetensors_dir(mc, cfgE.model, **kw)
        if cfgE.weights == "gguf":
            from b200serve.models.gguf import load_gguf_quantized, load_gguf_weights
            if dev.type == "cuda":
                return load_gguf_quantized(mc, cfgE.model, **kw)
            return load_gguf_weights(mc, cfgE.model, **kw)
        raise ValueError(f"unknown weights source {cfgE.weights!r}")

    def _size_kv(self, mc, nkv_local, dtype, dev) -> int:
        cfgE = self.config
        esz = torch.tensor([], dtype=dtype).element_size()
        per_block = KVCache.bytes_per_block(_kv_layers(mc), nkv_local, mc.head_dim, esz, cfgE.kv_format)
        if cfgE.kv_format == "turboquant" and cfgE.kv_boundary_layers > 0:    # bf16 boundary layers
            per_block += KVCache.bytes_per_block(min(_kv_layers(mc), 2 * cfgE.kv_boundary_layers), nkv_local,
                                                 mc.head_dim, esz, "bf16")
        state = 0
        if cfgE.kv_format == "turboquant" and cfgE.kv_residual_tokens > 0:   # bf16 residual-window pages
            rw = (cfgE.kv_residual_tokens + BLOCK - 1) // BLOCK * BLOCK
            state += _window_pages(cfgE.max_batch, rw) * KVCache.bytes_per_block(_kv_layers(mc), nkv_local,
                                                                                mc.head_dim, esz, "bf16")
        if mc.is_hybrid:
            from b200serve.models.hybrid import LinearState
            state = (cfgE.max_batch + 1) * LinearState.bytes_per_slot(mc, cfgE.tp_size)
        want = cfgE.max_batch * ((cfgE.max_seq + BLOCK - 1) // BLOCK) + 64
        if cfgE.kv_blocks:
            return cfgE.kv_blocks
        if dev.type == "cuda":
            free, _ = torch.cuda.mem_get_info(dev)
            budget = int((free - (6 << 30) - state) * cfgE.kv_mem_fraction)
            n = max(64, budget // per_block)
            return int(min(n, want))
        return int(min(want, 4096))

    def unload(self, status_callback=None):
        self.stop_loop()
        if self.runner is not None:
            inner = getattr(self.runner, "inner", self.runner)
            inner.release_graphs()
        self.runner = self.scheduler = self.kv = self.weights = None
        if torch.cuda.is_available():
            torch.cuda.empty_cache()

    def periodic_cleanup(self):
        if torch.cuda.is_available() and self.scheduler is not None and not self.scheduler.has_work():
            torch.cuda.empty_cache()

    def get_context_size(self) -> int:
        return self.config.max_seq

    def count_tokens(self, text: str) -> int:
        if self.tokenizer is None:
            return len(text) // 4
        return len(self.tokenizer.encode(text, add_special_tokens=False))

    def metrics(self) -> dict:
        return self.scheduler.metrics() if self.scheduler else {}

    # ------------------------------------------------------------ loop thread
    def start_loop(self):
        if self._thread is not None:
            return
        self._stop.clear()
        self._thread = threading.Thread(target=self._loop, name="b200-engine", daemon=True)
        self._thread.start()
        if self.config.step_timeout_s > 0 and self._watch is None:
            self._watch = threading.Thread(target=self._watchdog, name="b200-watchdog", daemon=True)
            self._watch.start()

    def stop_loop(self):
        if self._thread is None:
            return
        self._stop.set()
        with self._wake:
            self._wake.notify_all()
        self._thread.join(timeout=30)
        self._thread = None
        if self._watch is not None:
            self._watch.join(timeout=5)
            self._watch = None
        if self.world > 1 and hasattr(self.runner, "shutdown_workers"):
            self.runner.shutdown_workers()

    def _loop(self):
        if self.device.type == "cuda":
            torch.cuda.set_device(self.device)
        while not self._stop.is_set():
            if not self.scheduler.has_work():
                with self._wake:
                    self._wake.wait(timeout=0.05)
                continue
            try:
                self._step_t0 = time.monotonic()
                self.scheduler.step()
                self._step_t0 = None
                self.stalled = False
            except Exception as e:  # fail every in-flight request, keep the loop alive
                self._step_t0 = None
                _log.exception("engine step failed")
                self._error = e
                for r in list(self.scheduler.running) + list(self.scheduler.waiting):
                    r.aborted = True
                    self.scheduler._finish(r, "error")
                self.scheduler.running.clear()
                self.scheduler.waiting.clear()

    def _watchdog(self):
        """Per-request watchdog: when one forward step runs past ``step_timeout_s`` (a hung
        collective or kernel), every request it holds is finished with an error so that its
        client is released, and the engine reports itself stalled. The scheduler's lists are
        left alone: if the step ever returns, the loop drops the aborted requests normally."""
        limit = self.config.step_timeout_s
        flagged = None
        while not self._stop.is_set():
            self._stop.wait(min(1.0, limit / 4))
            t0 = self._step_t0
            if t0 is None or t0 == flagged or time.monotonic() - t0 < limit:
                continue
            flagged = t0
            self.stalled = True
            self._error = RuntimeError(f"engine step exceeded {limit:.0f} s")
            _log.error("b200: engine step exceeded %.0f s; failing its requests", limit)
            sched = self.scheduler
            for r in list(sched.running) + list(sched.waiting):
                r.aborted = True
                if r.state != "finished":
                    r.state, r.finish_reason = "finished", "error"
                    r.finish_time = time.perf_counter()
                    r.done_event.set()

    def submit(self, req: Request) -> Request:
        self.load()
        self.start_loop()
        self.scheduler.add(req)
        with self._wake:
            self._wake.notify_all()
        return req

    # ------------------------------------------------------------ batch API
    def generate(self, prompts, params: SamplingParams = None, timeout: float = None):
        """Token-id prompts -> finished Requests (output ids, ttft, finish_reason)."""
        params = params or SamplingParams()
        stop_ids = set() if params.ignore_eos else self.tokenizer.stop_ids
        reqs = [self.submit(Request(prompt=list(p), params=params, stop_ids=stop_ids)) for p in prompts]
        for r in reqs:
            if not r.done_event.wait(timeout):
                raise TimeoutError(f"{r.rid} did not finish")
        return reqs

    def embed(self, texts, timeout: float = 600.0):
        """Mean-pooled final hidden states (after the final RMSNorm) of each text, computed by
        this engine's model in its scheduler loop. Returns (vectors, token counts)."""
        self.load()
        self.start_loop()
        reqs = []
        for t in texts:
            ids = self.tokenizer.encode(t if isinstance(t, str) else str(t), add_special_tokens=False) or [0]
            ids = ids[: self.config.max_seq - 1]
            reqs.append(self.scheduler.add_embedding(Request(prompt=ids, params=SamplingParams(max_tokens=1))))
        with self._wake:
            self._wake.notify_all()
        for r in reqs:
            if not r.done_event.wait(timeout):
                raise TimeoutError("embedding request did not finish")
            if r.embedding is None:
                raise RuntimeError("embedding failed: " + str(self._error or "engine error"))
        return [r.embedding for r in reqs], [len(r.tokens) for r in reqs]

    # ------------------------------------------------------------ BaseEngine
    def _fit_prompt(self, messages, max_tokens, enable_thinking, tools):
        """Chat template -> token ids that fit the context with room for ``max_tokens``.

        A conversation that does not fit is compacted and trimmed by ``ensure_context_fit``
        (the reference's pre-flight, core/inference.py ensure_context_fit) and the result is
        reported as the ``context_fit`` stat (the API's ``x_context_fit``). A prompt that still
        leaves no room for one completion token raises ValueError: the head of the prompt
        (the system prompt) is never dropped silently."""
        ctx = self.config.max_seq
        tmpl = lambda msgs: self.tokenizer.apply_chat_template(msgs, add_generation_prompt=True,
                                                               enable_thinking=enable_thinking, tools=tools)
        prompt = tmpl(messages)
        fit = None
        if len(prompt) + min(max_tokens, ctx // 4) > ctx:
            from b200serve.core.inference import ensure_context_fit
            messages, fit = ensure_context_fit(messages, ctx, min(max_tokens, ctx // 4),
                                               count_fn=self.count_tokens)
            prompt = tmpl(messages)
            fit = dict(fit, prompt_tokens=len(prompt))
        if len(prompt) >= ctx:
            raise ValueError(f"prompt of {len(prompt)} tokens does not fit the {ctx}-token context "
                             f"even after compaction; shorten the conversation")
        return prompt, fit

    def generate_streaming(self, messages, max_tokens, temperature, on_token=None, on_complete=None,
                           enable_thinking=True, grammar=None, response_format=None, raw_output=False,
                           web_tools=False, reasoning_effort=None, on_telemetry=None, sampling=None,
                           tools=None, images=None) -> str:
        self.load()
        params = SamplingParams.from_dict(sampling, temperature=temperature,
                                          max_tokens=max_tokens if max_tokens and max_tokens > 0 else 8192)
        prompt, fit = self._fit_prompt(messages, params.max_tokens, enable_thinking, tools)
        mm = None
        if images:
            prompt, mm = self.prepare_images(prompt, images)
            if len(prompt) >= self.config.max_seq:
                raise ValueError(f"prompt with images is {len(prompt)} tokens; the context is {self.config.max_seq}")
        if len(prompt) + params.max_tokens > self.config.max_seq:
            params.max_tokens = self.config.max_seq - len(prompt)
        # the reference halts at once on a faked conversational turn (STOP_STRINGS, applied by
        # core/engine_transformers.py:1255 through StopStringCriteria) and on the request's stops
        stop_strings = [s for s in list(STOP_STRINGS) + list(params.stop) if s]
        hold = max((len(s) for s in stop_strings), default=0) + 8
        q = queue.Queue()
        dec = IncrementalDecoder(self.tokenizer)
        text_so_far = [""]
        stopped_by = [None]

        def _cb(req, tok):
            delta = dec.push(tok)
            if tok in req.stop_ids:
                delta = ""
            q.put(("tok", delta))
            if delta and stop_strings:
                text_so_far[0] += delta
                tail = text_so_far[0][-(len(delta) + hold):]
                for s_ in stop_strings:
                    if s_ in tail:
                        stopped_by[0] = s_
                        return True
                text_so_far[0] = text_so_far[0][-4 * hold:]
            return False

        t_start = time.perf_counter()
        cap = None
        if on_telemetry is not None:
            if self.world > 1:
                raise NotImplementedError("forward telemetry runs on a single-rank engine")
            from b200serve.core.forward_telemetry import TelemetryCapture
            cap = TelemetryCapture(self.tokenizer)
        req = Request(prompt=prompt, params=params, stop_ids=self.tokenizer.stop_ids, on_token=_cb)
        req.telemetry = cap
        req.mm = mm
        req = self.submit(req)
        full, t_first, callback_error = "", None, None
        try:
            while True:
                try:
                    kind, delta = q.get(timeout=0.1)
                except queue.Empty:
                    if req.done_event.is_set() and q.empty():
                        break
                    continue
                if cap is not None:
                    for frame in cap.drain():
                        on_telemetry(frame)
                if delta:
                    if t_first is None:
                        t_first = time.perf_counter()
                    full += delta
                    if on_token:
                        on_token(delta)
        except BaseException as e:  # the consumer raised: abort generation, re-raise after cleanup
            callback_error = e
            self.scheduler.abort(req)
            req.done_event.wait(30)
        if cap is not None:
            for frame in cap.drain():
                on_telemetry(frame)
        t_end = time.perf_counter()
        n = len(req.output)
        wall = t_end - t_start
        ttft = (t_first - t_start) if t_first else (req.ttft or 0.0)
        dec_time = (t_end - t_first) if t_first else wall
        self._last_gen_stats = {
            "tokens": n, "prompt_tokens": len(prompt), "completion_tokens": n,
            "finish_reason": req.finish_reason if req.finish_reason in ("length", "stop") else "stop",
            "wall_time": round(wall, 2), "tok_per_sec": round(n / wall, 1) if wall > 0 else 0,
            "ttft": round(ttft, 3), "decode_tok_per_sec": round(max(n - 1, 0) / dec_time, 1) if dec_time > 0 else 0,
            "prefix_hit_tokens": req.prefix_hit,
        }
        if stopped_by[0] is not None:
            self._last_gen_stats["stop_string"] = stopped_by[0]
        if fit is not None:
            self._last_gen_stats["context_fit"] = fit
        if callback_error is not None:
            raise callback_error
        if self._error is not None and req.finish_reason == "error":
            err, self._error = self._error, None
            raise err
        clean = strip_think_blocks(full) if raw_output else _clean_response(full)
        if on_complete:
            on_complete(clean)
        return clean
