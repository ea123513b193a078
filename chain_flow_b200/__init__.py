"""chain_flow_b200: a B200-native (sm_100a) drafting engine for the chain-flow speculative decoder.

The Python surface mirrors the reference's drafting path (FlowDrafterProposer with
propose()/_beam_chains()/_beam_tree(), the shortlist file format, the drafter checkpoint
layout); everything numeric runs in hand-written CUDA kernels in libcfb.so, reached through the
C ABI declared in include/cfb.h. There is no CPU fallback.
"""
from ._lib import CfbError, load as load_library

__all__ = ["CfbError", "load_library"]
