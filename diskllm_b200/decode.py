"""Device-side decode loop for one sequence: the step sequence of DiskLLM's
diskllm_sample_grammar (src/core/sampler_api.c:48-73) -- mask, presence, repetition, sample --
followed by appending the sampled id to the history the next step penalises, all on the GPU.
The whole run of steps is captured once as a CUDA graph and replayed, so a step costs the
kernels' time and no host round trip.

The logits of step i are row i % R of a device ring (a real model writes them in place each step;
here they are given), the uniform of step i is uniforms[i] (one U[0,1) per step).
"""
from __future__ import annotations

import torch

from . import capi


class DecodeLoop:
    def __init__(self, logits_ring: torch.Tensor, uniforms: torch.Tensor, params: dict,
                 history: torch.Tensor, cap: int | None = None, mask_ring: torch.Tensor | None = None):
        assert logits_ring.is_cuda and logits_ring.dim() == 2
        self.dev = logits_ring.device
        self.ring = logits_ring
        self.mask_ring = mask_ring
        self.u = uniforms
        self.steps = uniforms.numel()
        self.params = params
        self.init_hist = history.to(self.dev, torch.int32).contiguous()
        self.cap = int(cap if cap is not None else self.init_hist.numel() + self.steps)
        assert self.cap >= self.init_hist.numel()
        self.hist_ids = torch.zeros(self.cap, dtype=torch.int32, device=self.dev)
        self.hist_off = torch.zeros(2, dtype=torch.int64, device=self.dev)
        self.init_off = torch.tensor([0, self.init_hist.numel()], dtype=torch.int64, device=self.dev)
        self.tokens = torch.empty(self.steps, dtype=torch.int32, device=self.dev)
        # scratch given to every call, so that nothing is allocated inside a capture
        nb = capi.workspace_bytes(self.ring[:1], self.u[:1], params, hist_ids=self.hist_ids, hist_off=self.hist_off,
                                  hist_max=self.cap)
        self.ws = torch.empty(max(nb, 256), dtype=torch.uint8, device=self.dev)
        self.graph = None

    def _reset(self):
        self.hist_ids[: self.init_hist.numel()].copy_(self.init_hist)
        self.hist_off.copy_(self.init_off)

    def _step(self, i: int):
        r = i % self.ring.shape[0]
        kw = {}
        if self.mask_ring is not None:
            kw["mask"] = self.mask_ring[r:r + 1]
        capi.sample_batch(self.ring[r:r + 1], self.u[i:i + 1], self.params, hist_ids=self.hist_ids,
                          hist_off=self.hist_off, hist_max=self.cap, token=self.tokens[i:i + 1],
                          workspace=self.ws, **kw)
        rc = capi.load_library().dllm_cuda_append_history(
            self.tokens[i:i + 1].data_ptr(), self.hist_ids.data_ptr(), self.hist_off.data_ptr(), self.cap,
            torch.cuda.current_stream(self.dev).cuda_stream)
        if rc != capi.DLLM_OK:
            raise capi.DllmError(f"dllm_cuda_append_history: {capi.STATUS_NAMES.get(rc, rc)}")

    def run_eager(self) -> torch.Tensor:
        """Every step launched from the host."""
        self._reset()
        for i in range(self.steps):
            self._step(i)
        return self.tokens

    def capture(self):
        """Records reset + all steps as one CUDA graph (after one eager step, which fixes the
        launch configuration outside the capture)."""
        self._reset()
        self._step(0)
        torch.cuda.synchronize(self.dev)
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph):
            self._reset()
            for i in range(self.steps):
                self._step(i)
        return self

    def replay(self) -> torch.Tensor:
        if self.graph is None:
            self.capture()
        self.graph.replay()
        return self.tokens
