"""Connector metadata carries every field the reference's scheduler side fills in
(metadata.py:74-92 in the reference's origami package)."""
import dataclasses

from origami_b200.metadata import OrigamiConnectorMetadata, OrigamiRestoreRequest, OrigamiSaveRequest


def test_connector_metadata_fields_and_defaults():
    fields = {f.name: f for f in dataclasses.fields(OrigamiConnectorMetadata)}
    assert list(fields) == ["reqs_to_restore", "reqs_to_save", "gpu_lossless_ratio", "fused_request_ids",
                            "fused_query_start_positions", "fused_query_token_counts", "fused_request_indices",
                            "fused_codecs", "fused_prefix_lengths"]
    m = OrigamiConnectorMetadata()
    assert m.gpu_lossless_ratio == 0 and m.fused_request_ids == ()
    for name in ("reqs_to_restore", "reqs_to_save", "fused_query_start_positions", "fused_query_token_counts",
                 "fused_request_indices", "fused_codecs", "fused_prefix_lengths"):
        assert getattr(m, name) == {}
    assert OrigamiConnectorMetadata().fused_codecs is not m.fused_codecs  # no shared defaults


def test_requests_keep_the_reference_fields():
    r = OrigamiRestoreRequest("r", "k", ((1, 2),), 20)
    assert (r.lossless_path, r.metric_request_id) == ("cpu", None)
    s = OrigamiSaveRequest("r", "k", ((1, 2),), 20)
    assert s.token_start == 0
