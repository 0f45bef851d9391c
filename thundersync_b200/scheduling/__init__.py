"""scheduling"""
