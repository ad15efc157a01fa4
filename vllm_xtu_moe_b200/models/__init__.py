"""Model families, configs and weights."""
