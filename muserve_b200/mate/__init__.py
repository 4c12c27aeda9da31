"""Drop-ins for the two ``mate`` vendor ops the reference's MoE path calls."""
