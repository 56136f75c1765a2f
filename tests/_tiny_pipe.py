"""A minimal pipeline with the hooks of diffusers' FluxPipeline that the
sampling wrapper replaces (prepare_latents, _unpack_latents) around a
transformer, with a deterministic per-token Euler loop; used by the sampling
layout tests."""

from __future__ import annotations

import torch


class Scheduler:
    def __init__(self, stochastic=False):
        self.config = {"stochastic_sampling": stochastic}


class Output:
    def __init__(self, images):
        self.images = images


class TinyPipe:
    def __init__(self, transformer, grid, text_tokens, text_dim=64, pooled_dim=32, device="cuda"):
        self.transformer, self.grid, self.scheduler = transformer, grid, Scheduler()
        g = torch.Generator().manual_seed(8)
        self.text = torch.randn(1, text_tokens, text_dim, generator=g).to(torch.bfloat16).to(device)
        self.pooled = torch.randn(1, pooled_dim, generator=g).to(torch.bfloat16).to(device)
        self.txt_ids = torch.zeros(text_tokens, 3, dtype=torch.int64, device=device)
        self.device = device

    def prepare_latents(self, seed):
        from hilberta_b200.flux_model import image_ids

        g = torch.Generator().manual_seed(seed)  # noise drawn in raster order
        lat = torch.randn(1, self.grid * self.grid, 64, generator=g).to(torch.bfloat16).to(self.device)
        return lat, image_ids(self.grid, self.device)

    def _unpack_latents(self, latents):
        return latents.reshape(latents.shape[0], self.grid, self.grid, latents.shape[-1])

    def __call__(self, steps=3, seed=0, output_type="image", callback_on_step_end=None):
        latents, ids = self.prepare_latents(seed)
        for i in range(steps):
            t = 1.0 - i / steps
            v = self.transformer(hidden_states=latents, encoder_hidden_states=self.text, pooled_projections=self.pooled,
                                 timestep=torch.tensor([t], device=self.device), img_ids=ids, txt_ids=self.txt_ids,
                                 guidance=torch.tensor([3.5], device=self.device)).sample
            latents = (latents.float() - v.float() / steps).to(latents.dtype)  # per-token update
            if callback_on_step_end is not None:
                callback_on_step_end(self, i, t, {"latents": latents})
        if output_type == "latent":
            return Output(latents)
        return Output(self._unpack_latents(latents))
