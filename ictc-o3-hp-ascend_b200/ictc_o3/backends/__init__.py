"""Execution backends; this distribution ships the CUDA (sm_100a) backend only."""
