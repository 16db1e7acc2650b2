"""complexity_framework_b200 package (populated below)."""
