"""belt_b200: the latent-KV decode hot path of BELT, written for B200 (sm_100a).

Modules:
  latent_format   the latent export directory: reader (``load_latent_layers``), writer, row layout
  layer           ``LatentLayer`` and ``derive_latent_tensors`` (load-time constants)
  decode          split-KV schedule, decode kernel, segment merge (``vllm_lrkv.cute_decode`` surface)
  latent_ops      absorbed query, V up-projection, cache write (``vllm_lrkv.latent_ops`` surface)
  latent_backend  the ``LRKV_LATENT`` attention backend (``vllm_lrkv.latent_backend`` surface)
  ops             every kernel entry point as a torch custom op (``torch.ops.lrkv_b200.*``)
  vllm_plugin     the vLLM plugin entry point, vLLM type bindings and the hybrid KV-cache hooks
  model           the attention block of a compressed layer (q_gate GEMM, q-norm / RoPE, gate, o_proj)
  kv_cache        hybrid KV-cache block size and layer grouping arithmetic
  dp              data-parallel partitioning of sequences across GPUs
  synth           seeded synthetic workloads of the benchmark configurations
  build           in-tree nvcc build of ``libbelt_b200.so``

The CUDA library is loaded on first use; without it every operator raises.
"""

__version__ = "0.1.0"
