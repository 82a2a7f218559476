"""Operational checks and planning CLIs (``python -m libra_b200.infra.preflight <command>``)."""
