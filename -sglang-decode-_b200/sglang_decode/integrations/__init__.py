"""Serving-framework integrations (SGLang v0.4.6.post5 attention backend)."""
