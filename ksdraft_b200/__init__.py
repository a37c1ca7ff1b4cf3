"""ksdraft_b200 — B200 (sm_100a) INT8 hot path of KSDraft behind its operator API.

Modules mirror the reference package layout for the path:
  ksdraft_b200.kernels   quantize_last_dim, dequantize_last_dim, w8a8_gemm,
                         Int8Linear, KS3Int8Cell/_KS3Int8Train, project_fused
  ksdraft_b200.model     _match_payload_sign, RosaMixer, the vocab-sharded LM head
  ksdraft_b200.train     quantize_last_dim_dithered, data-parallel step helpers
  ksdraft_b200.install   rebinds those names inside an importable `ksdraft`
All compute runs in libksd8.so (hand-written sm_100a CUDA behind a C ABI).
"""

__version__ = "0.1.0"
