"""Utilities: flat parameter storage, timing, clock sampling."""
