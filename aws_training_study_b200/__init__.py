"""B200-native prefill context-parallel (PCP) history attention.

``aws_training_study_b200.pcp_attention`` mirrors the reference's
``pcp_attention`` host API (config, striped layout, KV packing) and runs the
attention on hand-written sm_100a CUDA (TMA + tcgen05/TMEM) behind the C ABI
in ``include/pcp_attn.h``; the KV ring between ranks is NCCL send/recv on a
high-priority stream.
"""

__version__ = "0.1.0"
