"""Child process of tests/test_vllm_backend_gpu.py: a vLLM engine (in-process engine core) on a
tiny random-weight Llama model with the LSSA-B8 backend, a few prompts of ragged lengths decoded
greedily; every attention call of every layer is recorded in the row-replay verifier's format
and saved with torch.save.

    python tests/vllm_run.py OUT.pt [--sink]
"""
import json
import os
import sys
import tempfile

os.environ.setdefault("VLLM_ENABLE_V1_MULTIPROCESSING", "0")
ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)

import torch  # noqa: E402

H, KVH, DH, LAYERS = 8, 2, 128, 2
PROMPT_LENS = (200, 77, 128)
NEW_TOKENS = 6


def tiny_llama(path):
    cfg = dict(architectures=["LlamaForCausalLM"], model_type="llama", hidden_size=H * DH, intermediate_size=1024,
               num_attention_heads=H, num_key_value_heads=KVH, head_dim=DH, num_hidden_layers=LAYERS, vocab_size=512,
               max_position_embeddings=1024, rms_norm_eps=1e-5, rope_theta=10000.0, torch_dtype="bfloat16",
               tie_word_embeddings=False, bos_token_id=1, eos_token_id=2)
    with open(os.path.join(path, "config.json"), "w") as f:
        json.dump(cfg, f)


def main():
    out_path = sys.argv[1]
    sink = "--sink" in sys.argv
    from lockstep_b200 import vllm_backend as VB
    VB.register(sink=sink)
    VB.DUMP = []
    from vllm import LLM, SamplingParams
    with tempfile.TemporaryDirectory() as d:
        tiny_llama(d)
        llm = LLM(model=d, load_format="dummy", skip_tokenizer_init=True, enforce_eager=True, dtype="bfloat16",
                  block_size=16, max_model_len=512, max_num_seqs=4, max_num_batched_tokens=2048,
                  num_gpu_blocks_override=256, enable_prefix_caching=False, gpu_memory_utilization=0.15,
                  attention_config={"backend": "CUSTOM"}, compilation_config={"mode": 0}, seed=0)
        g = torch.Generator().manual_seed(0)
        prompts = [{"prompt_token_ids": torch.randint(3, 500, (n,), generator=g).tolist()} for n in PROMPT_LENS]
        outs = llm.generate(prompts, SamplingParams(max_tokens=NEW_TOKENS, temperature=0.0, ignore_eos=True))
        tokens = [list(o.outputs[0].token_ids) for o in outs]
    torch.save(dict(dump=VB.DUMP, tokens=tokens, sink=sink, H=H, KVH=KVH, DH=DH), out_path)
    print("steps recorded:", len(VB.DUMP), "tokens:", tokens)


if __name__ == "__main__":
    main()
