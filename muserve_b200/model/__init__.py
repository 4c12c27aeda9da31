"""Model-layer entry points of the MoE path (``muserve/model``)."""
