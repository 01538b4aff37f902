"""Runtime: model runner (buffers, CUDA graphs), scheduler, sampler, engine."""
