"""Times the reference's own end-to-end decode loop on the TinyLlama-1.1B
architecture: ``metagross.generate_llama.generate_tinyllama_fused`` of the
unmodified reference installed in baseline/_ref, on a random-init Hugging Face
``LlamaForCausalLM`` of that architecture (22 layers, hidden 2048, 32 q / 4 kv
heads, FFN 5632, vocab 32000, fp16) with a stub tokenizer that hands out
seeded random prompt ids (no checkpoint or tokenizer files offline).  The
reference decodes one sequence per call, so a stated number of sequences run
one after another.  Prints one JSON line.

Run in a fresh interpreter whose import path holds baseline/_ref and not this
repository (bench.py does that): the reference's package is also named
``metagross``.

    python baseline/time_reference_decode.py [--sequences S] [--new-tokens N]
"""
import argparse
import json
import time

import torch


class StubTokenizer:
    """Returns the given prompt ids for any prompt; decodes ids to a string."""

    class _Enc:
        def __init__(self, ids):
            self.input_ids = ids

    def __init__(self, ids):
        self.ids = ids

    def __call__(self, prompt, return_tensors="pt"):
        return self._Enc(self.ids)

    def decode(self, ids):
        return " ".join(str(int(i)) for i in ids)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--sequences", type=int, default=2)
    ap.add_argument("--new-tokens", type=int, default=64)
    ap.add_argument("--prompt-len", type=int, default=128)
    a = ap.parse_args()
    from transformers import LlamaConfig, LlamaForCausalLM

    from metagross.generate_llama import generate_tinyllama_fused  # the reference's own loop

    cfg = LlamaConfig(hidden_size=2048, intermediate_size=5632, num_hidden_layers=22, num_attention_heads=32,
                      num_key_value_heads=4, vocab_size=32000, max_position_embeddings=2048, rms_norm_eps=1e-5,
                      rope_theta=10000.0, torch_dtype=torch.float16)
    torch.manual_seed(1234)
    with torch.device("cuda"):
        model = LlamaForCausalLM(cfg).to(torch.float16)
    model.eval()
    g = torch.Generator().manual_seed(1234)
    prompts = torch.randint(0, cfg.vocab_size, (a.sequences, a.prompt_len), generator=g)
    # warm-up: one short sequence (cuBLAS, kernel loading)
    generate_tinyllama_fused(model, StubTokenizer(prompts[:1].cuda()), "", max_new_tokens=4)
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    for s in range(a.sequences):
        generate_tinyllama_fused(model, StubTokenizer(prompts[s:s + 1].cuda()), "", max_new_tokens=a.new_tokens)
    torch.cuda.synchronize()
    el = time.perf_counter() - t0
    toks = a.sequences * a.new_tokens
    print(json.dumps({"metric": "decode tokens/s", "value": round(toks / el, 2), "unit": "tokens/s",
                      "impl": "reference generate_tinyllama_fused (baseline/_ref)",
                      "sample": f"{a.sequences} sequences x {a.new_tokens} new tokens, prompts of {a.prompt_len} "
                                f"seeded random ids, one sequence per call, serially; wall {el:.2f} s including "
                                f"each call's prefill", "seconds": round(el, 3)}))


if __name__ == "__main__":
    main()
