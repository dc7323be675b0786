"""Data-parallel plumbing: process groups, gradient synchronisation, collectives."""
