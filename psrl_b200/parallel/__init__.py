"""Parallelism: process groups, sharded DP, tensor/expert parallel, peer-memory transfers."""
