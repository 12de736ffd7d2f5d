"""The refiner's autoregressive chunk loop on the B200 model.

Mirrors ``CausalInferencePipeline.inference_sr``'s hot loop
(video_refiner/pipeline_sr/causal_inference.py:858-976) for the shipped
1-step schedule: per 3-latent-frame chunk,
  1. optional LQ-anchor harvest: the LR chunk's frames run as independent
     1-frame forwards with no cache; their per-layer roped K / V become the
     anchor (causal_inference.py:426-508);
  2. denoise: one forward at t = 625 over the rolling cache (+ anchor), then
     x0 = x_t - (t/1000) * flow in fp64 (utils/sr_dit_wrapper.py:551-558);
  3. KV refresh: one forward over x0 at t = context_noise (0) that writes the
     chunk's K / V into the cache, which keeps the newest ``kv_len`` frames.

The harvest of chunk i + 1 reads only chunk i + 1's LR frames (and the text
context), not the cache, so ``step(..., next_lq_chunk=...)`` starts it on a
side stream before chunk i's forwards and the next step picks its K / V up:
on one GPU it fills the gaps between chunk i's kernels, and its result is the
one a serial harvest would give (its own scratch buffers, its own temporal
position word).
"""
from __future__ import annotations

import copy

import torch

from .model import KVRing, SRDiT


class RefinerStream:
    """Per-chunk refinement over a rolling KV cache.

    ``graphs=True`` replays each step from a CUDA graph: a step is keyed by the
    ring phase (slot of the oldest cached frame, cached frames) and the chunk
    shape; the first visit of a key runs eagerly (it also warms up lazily built
    state), the second captures the two forwards and the flow->x0 update, and
    later visits replay them. The temporal RoPE position is device-resident
    (``SRDiT.set_t_offset``), so one graph serves every chunk with the same ring
    phase -- in the steady state the phases repeat every (kv_len + chunk) /
    chunk chunks. Steps with an LQ anchor run eagerly.
    """

    def __init__(self, model: SRDiT, context: torch.Tensor, *, denoise_t: float = 625.0,
                 context_noise: float = 0.0, num_train_timesteps: int = 1000,
                 frame_tokens: int | None = None, graphs: bool = False):
        self.model = model
        self.denoise_t = float(denoise_t)
        self.context_noise = float(context_noise)
        self.ntt = num_train_timesteps
        self.cache: KVRing | None = None
        self.t_offset = 0
        self._frame_tokens = frame_tokens
        self.graphs = graphs
        self._graphs = {}
        self._seen = set()
        self.context = context.clone()   # static: graph replays read this buffer
        # text embedding + per-block cross K/V of the context, built once per
        # context (rebuilt in place when set_context changes it)
        self.text = None
        self._text_dirty = True
        # anchor harvest of the next chunk, started ahead on a side stream
        self._harvester = None
        self._side = None
        self._pending = None   # (t_offset, per-layer K / V, completion event or None)

    def set_context(self, context: torch.Tensor):
        """Replace the text context (copied into the step's static buffer)."""
        if context.shape != self.context.shape:
            self.context = context.clone()
            self.text = None
            self._graphs.clear()
            self._seen.clear()
        else:
            self.context.copy_(context)
        self._text_dirty = True

    def _ensure_text(self):
        if self._text_dirty:
            self.text = self.model.text_cache(self.context, into=self.text)
            self._text_dirty = False

    def reset(self):
        self.cache = None
        self.t_offset = 0
        self._pending = None

    def harvest_anchor(self, lq_chunk, harvest_t=0.0):
        """Per-frame anchor K / V: the LR chunk's frames as independent 1-frame
        samples (frame j at temporal position t_offset + j, no cache), run as one
        forward whose self-attention keeps every frame to itself -- the
        reference's batch of B = f samples (causal_inference.py:456-460)."""
        _, kv = self.model.forward_chunk(lq_chunk, harvest_t, self.context, cache=None,
                                         t_offset=self.t_offset, return_kv=True,
                                         text=self.text, independent_frames=True)
        return kv

    def _harvest_model(self):
        """The model with its own scratch buffers, temporal-position word, status
        word and per-shape caches (weights, RoPE tables and the text cache are
        shared), so a harvest on the side stream never touches a buffer that
        the main stream's forwards use."""
        if self._harvester is None:
            h = copy.copy(self.model)
            h._bufs = {}
            h._cross_plans = {}
            h._temb = {}
            h.status = torch.zeros_like(self.model.status)
            h.t_offset_dev = torch.zeros_like(self.model.t_offset_dev)
            h.graph_capture = False
            self._harvester = h
        return self._harvester

    def prefetch_anchor(self, lq_chunk, t_offset, harvest_t=0.0):
        """Start the anchor harvest of the chunk at temporal position ``t_offset``
        (its LR frames ``lq_chunk``) on a side stream; the ``step`` of that chunk
        takes the result (``causal_inference.py:878-899`` harvests each chunk
        from its LR frames alone). On a CPU model it runs at once."""
        self._ensure_text()
        dev = self.model.device
        if getattr(self.model, "world", 1) > 1:
            # a sharded model's harvest runs collectives, which every rank must
            # issue in one order on one stream: harvest in line instead
            self._pending = (t_offset, self.model.forward_chunk(
                lq_chunk, harvest_t, self.context, cache=None, t_offset=t_offset,
                return_kv=True, text=self.text, independent_frames=True)[1], None)
            return
        h = self._harvest_model()
        if dev.type != "cuda":
            _, kv = h.forward_chunk(lq_chunk, harvest_t, self.context, cache=None,
                                    t_offset=t_offset, return_kv=True, text=self.text,
                                    independent_frames=True)
            self._pending = (t_offset, kv, None)
            return
        main = torch.cuda.current_stream(dev)
        if self._side is None:
            self._side = torch.cuda.Stream(dev)
        side = self._side
        side.wait_stream(main)          # the LR frames, the text cache are ready
        lq_chunk.record_stream(side)    # the caller may drop it before the side reads it
        with torch.cuda.stream(side):
            _, kv = h.forward_chunk(lq_chunk, harvest_t, self.context, cache=None,
                                    t_offset=t_offset, return_kv=True, text=self.text,
                                    independent_frames=True)
            done = torch.cuda.Event()
            done.record(side)
        self._pending = (t_offset, kv, done)

    def _take_anchor(self, lq_chunk, harvest_t):
        """This chunk's anchor: the prefetched harvest if one was started for this
        temporal position, else a harvest now, on the main stream."""
        pend, self._pending = self._pending, None
        if pend is not None and pend[0] == self.t_offset:
            _, kv, done = pend
            if done is not None:
                main = torch.cuda.current_stream(self.model.device)
                main.wait_event(done)
                for k, v in kv:   # made on the side stream, read and freed on main
                    k.record_stream(main)
                    v.record_stream(main)
            return kv
        return self.harvest_anchor(lq_chunk, harvest_t)

    def check_status(self):
        """Raise if a kernel of the main or the harvest stream gave up on a wait."""
        self.model.check_status()
        if self._harvester is not None:
            self._harvester.check_status()

    def _ensure_cache(self, noisy_chunk):
        if self.cache is None:
            m = self.model
            ph, pw = m.cfg.patch_size[1], m.cfg.patch_size[2]
            h, w = noisy_chunk.shape[2] // ph, noisy_chunk.shape[3] // pw
            self.cache = m.new_cache(h * w, grid_hw=(h, w))

    def _step_eager(self, noisy_chunk, lq_chunk=None, anchor_harvest_t=0.0, anchor=None):
        m = self.model
        if anchor is None and lq_chunk is not None:
            anchor = self.harvest_anchor(lq_chunk, anchor_harvest_t)
        flow = m.forward_chunk(noisy_chunk, self.denoise_t, self.context, cache=self.cache,
                               t_offset=self.t_offset, anchor_kv=anchor, text=self.text)
        sigma = self.denoise_t / self.ntt
        x0 = (noisy_chunk.double() - sigma * flow.double()).to(noisy_chunk.dtype)
        # the refresh pass only fills the ring: its prediction is discarded
        m.forward_chunk(x0, self.context_noise, self.context, cache=self.cache,
                        t_offset=self.t_offset, update_cache=True, text=self.text, kv_only=True)
        self.t_offset += noisy_chunk.shape[1]
        return x0

    def _capture(self, key, noisy_chunk):
        m = self.model
        inp = noisy_chunk.clone()
        saved = (self.cache.start, self.cache.frames, self.t_offset)
        graph = torch.cuda.CUDAGraph()
        m.graph_capture = True
        try:
            torch.cuda.synchronize(noisy_chunk.device)
            with torch.cuda.graph(graph):
                out = self._step_eager(inp)
        finally:
            m.graph_capture = False
            self.cache.start, self.cache.frames, self.t_offset = saved
        self._graphs[key] = (graph, inp, out)
        return self._graphs[key]

    def step(self, noisy_chunk: torch.Tensor, lq_chunk: torch.Tensor | None = None,
             anchor_harvest_t: float = 0.0, next_lq_chunk: torch.Tensor | None = None,
             next_t_offset: int | None = None):
        """Refine one chunk [C, f, H, W] (device, bf16); returns x0 [C, f, H, W] bf16
        (with graphs, a buffer the next replay of the same ring phase overwrites).

        ``lq_chunk``: this chunk's LR frames, for the LQ anchor (harvested now
        unless a previous step prefetched it). ``next_lq_chunk``: the next
        chunk's LR frames; their harvest starts on the side stream before this
        chunk's forwards, for temporal position ``next_t_offset`` (default: right
        after this chunk)."""
        self._ensure_cache(noisy_chunk)
        self._ensure_text()
        anchor = self._take_anchor(lq_chunk, anchor_harvest_t) if lq_chunk is not None else None
        if next_lq_chunk is not None:
            nt = self.t_offset + noisy_chunk.shape[1] if next_t_offset is None else next_t_offset
            self.prefetch_anchor(next_lq_chunk, nt, anchor_harvest_t)
        if not self.graphs or anchor is not None:
            return self._step_eager(noisy_chunk, anchor=anchor)
        key = (self.cache.start, self.cache.frames, tuple(noisy_chunk.shape))
        entry = self._graphs.get(key)
        if entry is None:
            if key not in self._seen:
                self._seen.add(key)
                return self._step_eager(noisy_chunk)
            entry = self._capture(key, noisy_chunk)
        graph, inp, out = entry
        self.model.set_t_offset(self.t_offset)
        inp.copy_(noisy_chunk)
        graph.replay()
        f = noisy_chunk.shape[1]
        self.cache.commit(f)
        self.t_offset += f
        return out


def sr_noise(lr_up: torch.Tensor, noise: torch.Tensor, sigma: float) -> torch.Tensor:
    """The refiner's starting latent: (1 - sigma) * upsampled LR + sigma * noise
    (causal_inference.py:667-668)."""
    return ((1.0 - sigma) * lr_up.float() + sigma * noise.float()).to(lr_up.dtype)


def refine_clip(stream: RefinerStream, noisy: torch.Tensor, chunk: int = 3,
                lq: torch.Tensor | None = None, events: list | None = None) -> torch.Tensor:
    """Every chunk of a clip's noisy latent [C, T, H, W] through ``stream`` (the
    loop of causal_inference.py:858-976), each chunk's LQ anchor harvested from
    the same frames of ``lq`` (the upsampled LR latent) when given, the next
    chunk's harvest started ahead. Returns the refined latent [C, T, H, W];
    ``events`` (a list) receives a CUDA event after each chunk."""
    T = noisy.shape[1]
    if T % chunk:
        raise ValueError(f"{T} latent frames are not whole {chunk}-frame chunks")
    outs = []
    for i in range(0, T, chunk):
        nxt = lq[:, i + chunk:i + 2 * chunk] if lq is not None and i + chunk < T else None
        out = stream.step(noisy[:, i:i + chunk],
                          lq_chunk=lq[:, i:i + chunk] if lq is not None else None,
                          next_lq_chunk=nxt)
        outs.append(out.clone() if stream.graphs else out)
        if events is not None:
            ev = torch.cuda.Event(enable_timing=True)
            ev.record()
            events.append(ev)
    return torch.cat(outs, dim=1)
