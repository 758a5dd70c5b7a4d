"""B200 paged split-KV ("PS") attention for prime-rl's vLLM inference path.

Modules (imported on demand; nothing is loaded at package import):

* ``ops``       -- torch-facing ops over libps_attn.so: KV append (16-bit and
  fp8), paged decode (split-KV, fused combine and append, cascade, fp8),
  chunked prefill (tcgen05), fused RoPE + append, the fp8 page gather.
* ``backend``   -- the vLLM attention backend (``register()``).
* ``sharding``  -- KV-head-sharded decode with the head all-gather over NVLink
  peer memory or NCCL; sequence-batch balancing.
* ``dcp``       -- decode context parallelism over peer memory.
* ``peer``      -- per-rank IPC slabs shared by ``dcp`` and ``sharding``.
* ``workloads`` -- the benchmark configurations' synthetic batches.
* ``_lib`` / ``_build`` -- the ctypes binding and the in-tree nvcc build.
"""
