"""Engine integrations of the B200 paged fused-MoE layer."""
