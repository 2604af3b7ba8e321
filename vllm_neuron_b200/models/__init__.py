"""Model zoo: GPT-OSS, Llama3 (+EAGLE3 draft), Qwen3-VL, Qwen3-Next, synthetic KV model."""
