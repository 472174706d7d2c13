"""Stand-ins for the few vLLM objects the connector reads.

Each carries only the attributes the connector (and the reference's
connector) uses: ``req_id``, ``block_ids``, ``num_computed_tokens``,
``num_scheduled_tokens``, ``finished_req_ids``, ``kv_transfer_params`` and the
model/cache/transfer config fields read in ``__init__``.
"""

from __future__ import annotations

from types import SimpleNamespace

BS = 16


def fake_config(extra=None, head_dim=128, cache_dtype="auto", rotary_factor=1.0):
    hf = SimpleNamespace(head_dim=head_dim, hidden_size=4096, num_attention_heads=32,
                         partial_rotary_factor=rotary_factor, rope_theta=1e6)
    return SimpleNamespace(
        kv_transfer_config=SimpleNamespace(kv_connector_extra_config=extra or {}),
        cache_config=SimpleNamespace(block_size=BS, cache_dtype=cache_dtype),
        model_config=SimpleNamespace(hf_text_config=hf),
    )


def request(rid, params, n_prompt):
    return SimpleNamespace(request_id=rid, kv_transfer_params=params, num_prompt_tokens=n_prompt)


def new_req(rid, blocks, computed):
    return SimpleNamespace(req_id=rid, block_ids=(list(blocks),), num_computed_tokens=computed)


def sched_output(new=(), cached=None, scheduled=None, finished=()):
    cached = cached or SimpleNamespace(req_ids=[], new_block_ids=[], num_computed_tokens=[])
    return SimpleNamespace(scheduled_new_reqs=list(new), scheduled_cached_reqs=cached,
                           num_scheduled_tokens=dict(scheduled or {}),
                           finished_req_ids=set(finished))


def forward_context():
    return SimpleNamespace(no_compile_layers={}, virtual_engine=0)
