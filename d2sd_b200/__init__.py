"""d2sd_b200 -- B200 (sm_100a) tree-verification hot path of D2-SD.

Public surface (mirrors the reference's call surface):
  CascadeGraphRunner            drop-in for model/cascade_graph.py
  single_prefill_with_kv_cache  FlashInfer-signature level-1 / level-2 attention
  merge_state_in_place          FlashInfer-signature state merge
  cascade_attention, CascadePlan, Request
                                plan/run form of the two-level verify attention
  verify, Verifier              greedy acceptance (generation/d3_generator.py:204-225)
  BatchVerifier                 the same for a batch of requests in one launch
  ShardedVerifier               vocabulary-sharded acceptance across GPUs (NVLink
                                exchange of the rows' bests inside the kernel)
  PagedKVCache                  paged target cache with the accepted-branch commit
  PagedKVPool                   many sequences in one page pool, batched commit
  cascade_verify_forward        generation/verification.py:cascade_verify_forward
                                on these kernels
  PeerExchange                  KV-head-sharded output all-gather done by kernel (b)'s
                                own NVLink stores (multi-GPU)

All compute runs in ``libd2sd.so`` (built by ``python -m d2sd_b200.build``);
importing a kernel entry point without it raises.
"""
from .accept import BatchVerifier, ShardedVerifier, Verifier, verify
from .cascade import CascadePlan, Request, cascade_attention, shared_trunk_map
from .flashinfer_compat import merge_state_in_place, single_prefill_with_kv_cache
from .kv_cache import PagedKVCache, PagedKVPool
from .runner import CascadeGraphRunner
from .sharding import PeerExchange, RecordExchange

__all__ = [
    "BatchVerifier",
    "CascadeGraphRunner",
    "CascadePlan",
    "PagedKVCache",
    "PagedKVPool",
    "PeerExchange",
    "RecordExchange",
    "Request",
    "ShardedVerifier",
    "Verifier",
    "cascade_attention",
    "merge_state_in_place",
    "shared_trunk_map",
    "single_prefill_with_kv_cache",
    "verify",
]


def __getattr__(name):
    if name == "cascade_verify_forward":
        from .verification import cascade_verify_forward
        return cascade_verify_forward
    raise AttributeError(name)
