"""Experimental autoregressive samplers."""
