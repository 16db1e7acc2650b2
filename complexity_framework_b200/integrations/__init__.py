"""Third-party integrations (HF Transformers)."""
