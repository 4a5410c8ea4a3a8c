"""The B200 serving engine: paged KV cache, scheduler, sampler, model runner."""
