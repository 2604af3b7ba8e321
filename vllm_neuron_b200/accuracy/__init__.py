"""Accuracy toolkit: tolerance checks, logit validation, tensor capture."""
