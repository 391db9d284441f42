"""Layout / bitpack ops and the host codec boundary (mirrors the reference's
origami.lossless package)."""
