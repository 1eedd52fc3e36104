"""Minimal use of the engine: chat-formatted prompts through ``LLM.generate``.

``MODEL_PATH=/models/Qwen3-8B python example.py`` (an HF Qwen3 checkpoint with its tokenizer).
Without a checkpoint, ``python example.py --synthetic`` runs a random-weight Qwen3-8B-shaped model
(token ids in, token ids out) to check that the installation works on the GPU.
"""
import os
import sys


def main():
    from llmserve_b200 import LLM, SamplingParams
    if "--synthetic" in sys.argv:
        import tempfile

        from llmserve_b200.models.synthetic import QWEN3_8B, write_config_only
        path = write_config_only(os.path.join(tempfile.gettempdir(), "llmserve_b200_example"), QWEN3_8B)
        llm = LLM(path, load_format="dummy", max_model_len=1024)
        out = llm.generate([[1, 2, 3, 4], list(range(100, 164))], SamplingParams(temperature=0.6, max_tokens=32))
        for o in out:
            print(o["token_ids"])
        llm.exit()
        return
    from transformers import AutoTokenizer
    path = os.path.expanduser(os.environ.get("MODEL_PATH", "~/models/Qwen3-8B/"))
    tokenizer = AutoTokenizer.from_pretrained(path)
    llm = LLM(path, tensor_parallel_size=int(os.environ.get("TP", "1")))
    prompts = [tokenizer.apply_chat_template([{"role": "user", "content": p}], tokenize=False, add_generation_prompt=True)
               for p in ("introduce yourself", "list all prime numbers within 100")]
    for prompt, output in zip(prompts, llm.generate(prompts, SamplingParams(temperature=0.6, max_tokens=256))):
        print(f"\nPrompt: {prompt!r}\nCompletion: {output['text']!r}")
    llm.exit()


if __name__ == "__main__":
    main()
