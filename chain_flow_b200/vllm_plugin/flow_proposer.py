"""Import-path twin of the reference's ``chain_flow.vllm_plugin.flow_proposer`` so a vLLM
``speculative_config={"method": "custom_class", "model": "chain_flow_b200.vllm_plugin.flow_proposer.FlowDrafterProposer"}``
selects the sm_100a engine."""
from chain_flow_b200.proposer import FlowDrafterProposer

__all__ = ["FlowDrafterProposer"]
