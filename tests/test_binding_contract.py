"""CPU: the binding's call surface against what the reference's PagedTalkerKV
passes to a custom binding_factory (recorded by tests/golden/make_golden.py
from the reference itself, executor/talker_kv.py:358-388, 485-533)."""

from __future__ import annotations

import dataclasses
import inspect

import torch


def test_factory_keywords_are_accepted(nqt, golden):
    params = inspect.signature(nqt.B200TalkerBinding.__init__).parameters
    required = {n for n, p in params.items() if p.default is inspect.Parameter.empty and n != "self"}
    for factory in golden("binding.pt")["factories"]:
        keys = set(factory["keys"])
        assert keys <= set(params), keys - set(params)
        assert required <= keys, required - keys
        assert factory["workspace_dtype"] == "torch.uint8"


def test_metadata_fields_match_the_reference(nqt, golden):
    fx = golden("binding.pt")
    ours = [f.name for f in dataclasses.fields(nqt.TalkerAttentionMetadata)]
    assert ours == fx["metadata_fields"]
    for call in fx["calls"]:
        assert call["fields"] == ours
        meta = nqt.TalkerAttentionMetadata(**{k: call[k] for k in call["fields"]})
        assert meta.paged_kv_indptr.dtype == torch.int32 and meta.position_ids.dtype == torch.long
    # one prefill binding (packed query metadata) then decode plans on another binding of the slot
    kinds = [(c["binding"], c["qo_indptr"] is not None) for c in fx["calls"]]
    assert kinds[0] == (0, True) and all(k == (1, False) for k in kinds[1:])
