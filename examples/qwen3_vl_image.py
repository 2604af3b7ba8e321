"""Image + text prompt with Qwen3-VL: one image placeholder per image in the prompt is
expanded to the image's token count; the vision tower runs once per image (encoder cache).

    python examples/qwen3_vl_image.py --model /models/Qwen3-VL-32B-Instruct --image cat.jpg --tp 8
"""

import argparse

from vllm_neuron_b200 import LLM, SamplingParams


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--model", required=True)
    ap.add_argument("--image", required=True)
    ap.add_argument("--tp", type=int, default=1)
    a = ap.parse_args()
    from PIL import Image  # noqa: PLC0415  (optional dependency)

    llm = LLM(model=a.model, tensor_parallel_size=a.tp, max_model_len=8192, kv_cache_dtype="fp8")
    tok = llm.get_tokenizer()
    msgs = [{"role": "user", "content": [{"type": "image"}, {"type": "text", "text": "Describe this image."}]}]
    ids = tok.apply_chat_template(msgs, add_generation_prompt=True, tokenize=True)
    out = llm.generate([{"prompt_token_ids": ids, "multi_modal_data": {"image": Image.open(a.image)}}],
                       SamplingParams(temperature=0, max_tokens=128))
    print(out[0].outputs[0].text)
    llm.shutdown()


if __name__ == "__main__":
    main()
