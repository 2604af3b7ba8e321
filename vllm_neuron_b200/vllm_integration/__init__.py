"""Running this framework inside vLLM's own engine (``vllm serve`` / ``vllm.LLM``).

The platform plugin (``vllm_neuron_b200.platform.B200Platform``) installs two classes into
vLLM's configuration, as the Trainium plugin installs its worker and scheduler
(``vllm_neuron/vllm/platform.py:322-325`` and ``:376-387``):

* ``worker.B200VllmWorker`` (``parallel_config.worker_cls``): one per GPU.  It builds this
  framework's engine worker (model, parallel groups, fused collectives, KV cache, decode CUDA
  graphs) and runs vLLM's ``SchedulerOutput`` through this framework's model runner: vLLM
  keeps tokenisation, the request queue, KV block allocation and prefix caching; the forward
  pass, sampling and every kernel are this framework's.
* ``scheduler.B200VllmScheduler`` / ``B200VllmAsyncScheduler``
  (``scheduler_config.scheduler_cls``): vLLM's scheduler with this framework's step policy,
  in which a step is either prefill work or a decode batch, so decode steps always replay
  the per-bucket CUDA graphs.
"""
