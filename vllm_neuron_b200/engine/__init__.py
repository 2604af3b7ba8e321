"""Engine: scheduler, KV block manager, model runner, worker, LLM API."""
