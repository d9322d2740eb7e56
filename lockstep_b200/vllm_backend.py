"""LSSA-B8 as a vLLM attention backend (vLLM 0.22, v1 engine), over the serving-engine seam.

The reference ships its engine as a vLLM plugin with its own attention backend
(paper/main.tex:846-860): every attention call of a decoder layer runs the contract, prompt rows
as LSSA-B8 prefill rows and generated rows as decode rows, and a sequence's role in a step comes
from the scheduler's prefill flag, never from its number of query rows (docs/SPEC.md:88-93).
This module is that backend on this library:

  * Lssab8AttentionBackend -- the backend class: a KV cache of 16-token pages
    [num_blocks, 2, 16, KVH, dh] (K and V of a page side by side), head sizes 64 and 128, decoder
    self-attention only, no CUDA graphs (the forward pass reads host-side metadata);
  * Lssab8MetadataBuilder -- per step: query_start_loc, seq_lens, the block table, slot_mapping,
    and CommonAttentionMetadata.is_prefilling (num_computed_tokens < num_prompt_tokens, the
    scheduler's prefill flag) as each sequence's role;
  * Lssab8AttentionImpl -- one per attention layer: writes the step's K/V into vLLM's cache and
    runs lockstep_b200.engine.Lssab8Attention on it (the int8 lattice shadowing the cache, with
    the cache's page ids).

    from lockstep_b200 import vllm_backend
    vllm_backend.register()               # vLLM's CUSTOM backend slot -> Lssab8AttentionBackend
    llm = vllm.LLM(model=..., attention_config={"backend": "CUSTOM"}, block_size=16,
                   enable_prefix_caching=False, ...)

A prompt chunk must start on a multiple of 128 tokens (the contract's chunk rule,
reference/lssab8_selftest.py:292-317): whole prompts in one step, or a scheduler that cuts chunks
on 128-token boundaries; a prefix-cache hit that starts a prompt elsewhere is refused (ValueError).
The score scale is the contract's 1/sqrt(head_size); a model with another scale, ALiBi, a sliding
window, soft-capping or KV sharing is refused (NotImplementedError).  B9.1 (the sink) is chosen
at registration.

Setting DUMP to a list records every step of every layer in the row-replay verifier's format
(lockstep_b200.verify_rows: layer, nseq, qsl, sl, bt0, q, k, v, out, pref), for checking an
engine run row by row.
"""
import math
import re
from dataclasses import dataclass

import torch

from vllm.config import get_current_vllm_config
from vllm.v1.attention.backend import (AttentionBackend, AttentionCGSupport, AttentionImpl,
                                       AttentionMetadataBuilder, AttentionType)
from vllm.v1.attention.backends.registry import AttentionBackendEnum, register_backend

from . import engine as E

SINK = False          # B9.1 sink_alone for every layer (set by register())
DUMP = None           # a list to record verifier dumps into, or None


def register(sink=False):
    """Register Lssab8AttentionBackend as vLLM's CUSTOM attention backend (select it with
    attention_config={"backend": "CUSTOM"}); sink=True runs B9.1 sink_alone."""
    global SINK
    SINK = bool(sink)
    register_backend(AttentionBackendEnum.CUSTOM, __name__ + ".Lssab8AttentionBackend")


@dataclass
class Lssab8Metadata:
    num_tokens: int
    query_start_loc: list
    seq_lens: list
    is_prefill: list
    block_table: torch.Tensor
    slot_mapping: torch.Tensor


class Lssab8MetadataBuilder(AttentionMetadataBuilder[Lssab8Metadata]):
    _cudagraph_support = AttentionCGSupport.NEVER

    def __init__(self, kv_cache_spec, layer_names, vllm_config, device):
        super().__init__(kv_cache_spec, layer_names, vllm_config, device)

    def build(self, common_prefix_len, common_attn_metadata, fast_build=False):
        cm = common_attn_metadata
        if cm.is_prefilling is None:
            raise RuntimeError("the step carries no prefill flags (CommonAttentionMetadata.is_prefilling); the role "
                               "of a sequence's rows is never taken from its query length")
        n = cm.num_reqs
        qsl = [int(x) for x in cm.query_start_loc_cpu[:n + 1].tolist()]
        return Lssab8Metadata(num_tokens=qsl[-1], query_start_loc=qsl,
                              seq_lens=[int(x) for x in cm.seq_lens[:n].cpu().tolist()],
                              is_prefill=[bool(x) for x in cm.is_prefilling[:n].tolist()],
                              block_table=cm.block_table_tensor[:n], slot_mapping=cm.slot_mapping[:qsl[-1]])


class Lssab8AttentionBackend(AttentionBackend):
    supported_dtypes = [torch.float16, torch.bfloat16]
    supported_kv_cache_dtypes = ["auto", "float16", "bfloat16"]
    forward_includes_kv_cache_update = True

    @staticmethod
    def get_supported_kernel_block_sizes():
        return [E.PAGE]

    @staticmethod
    def get_name():
        return "CUSTOM"

    @staticmethod
    def get_impl_cls():
        return Lssab8AttentionImpl

    @staticmethod
    def get_builder_cls():
        return Lssab8MetadataBuilder

    @staticmethod
    def get_kv_cache_shape(num_blocks, block_size, num_kv_heads, head_size, cache_dtype_str="auto"):
        if block_size != E.PAGE:
            raise ValueError("LSSA-B8 pages hold 16 tokens (block_size=16)")
        return (num_blocks, 2, block_size, num_kv_heads, head_size)

    @staticmethod
    def use_cascade_attention(*args, **kwargs):
        return False

    @classmethod
    def get_supported_head_sizes(cls):
        return [64, 128]

    @classmethod
    def supports_attn_type(cls, attn_type):
        return attn_type == AttentionType.DECODER

    @classmethod
    def supports_compute_capability(cls, capability):
        return capability.major == 10


def _layer_index(layer):
    m = re.findall(r"\d+", getattr(layer, "layer_name", "") or "")
    return int(m[0]) if m else 0


class Lssab8AttentionImpl(AttentionImpl):
    def __init__(self, num_heads, head_size, scale, num_kv_heads=None, alibi_slopes=None, sliding_window=None,
                 kv_cache_dtype="auto", logits_soft_cap=None, attn_type=AttentionType.DECODER,
                 kv_sharing_target_layer_name=None, **kwargs):
        if alibi_slopes is not None or sliding_window not in (None, -1) or logits_soft_cap:
            raise NotImplementedError("LSSA-B8 has no ALiBi, sliding window or soft-capping")
        if attn_type != AttentionType.DECODER or kv_sharing_target_layer_name is not None:
            raise NotImplementedError("LSSA-B8 runs decoder self-attention with its own KV cache")
        if abs(scale * math.sqrt(head_size) - 1.0) > 1e-6:
            raise NotImplementedError("the contract's score scale is 1/sqrt(head_size), the model asks %r" % scale)
        self.num_heads, self.head_size, self.scale = num_heads, head_size, scale
        self.num_kv_heads = num_kv_heads or num_heads
        self.kv_cache_dtype = kv_cache_dtype
        cfg = get_current_vllm_config()
        self.max_len = int(cfg.model_config.max_model_len)
        self.max_seqs = 2 * int(cfg.scheduler_config.max_num_seqs) + 8   # slots, reused least recently used
        self.sink = SINK
        self.attn = None

    def forward(self, layer, query, key, value, kv_cache, attn_metadata, output, output_scale=None,
                output_block_scale=None):
        if output_scale is not None or output_block_scale is not None:
            raise NotImplementedError("fused output quantisation")
        if attn_metadata is None:                        # the engine's profiling run
            return output.fill_(0)
        md = attn_metadata
        n = md.num_tokens
        if self.attn is None:                            # the lattice shadows the cache: same page ids
            self.attn = E.Lssab8Attention(self.num_heads, self.num_kv_heads, self.head_size, kv_cache.shape[0],
                                          self.max_len, self.max_seqs, num_layers=1, sink=self.sink,
                                          device=query.device)
        k_cache, v_cache = kv_cache.unbind(1)
        meta = E.StepMeta(query_start_loc=md.query_start_loc, seq_lens=md.seq_lens, block_table=md.block_table,
                          slot_mapping=md.slot_mapping, is_prefill=md.is_prefill)
        q, k, v = query[:n], key[:n], value[:n]
        self.attn.forward(0, q, k, v, k_cache, v_cache, meta, out=output[:n])
        if DUMP is not None:
            DUMP.append(dict(layer=_layer_index(layer), nseq=len(md.seq_lens),
                             qsl=torch.tensor(md.query_start_loc), sl=torch.tensor(md.seq_lens),
                             bt0=md.block_table[:, 0].cpu(), q=q.cpu(), k=k.cpu(), v=v.cpu(),
                             out=output[:n].cpu(), pref=torch.tensor(md.is_prefill)))
        return output
