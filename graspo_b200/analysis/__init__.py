"""Post-run analysis and evaluation utilities (run as ``python -m graspo_b200.analysis.<tool>``)."""
